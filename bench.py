"""Benchmark of the B200 Gated DeltaNet hot path (one JSON line on rank 0).

Default workload: long batched chunk prefill, 64
independent sequences x 16 heads x 8192 tokens, chunk 64, k=v=128, bf16
q/k/v, fp32 g/beta/state/accumulation, bf16 core_attn_out. Synthetic seeded
inputs with config 0's distributions (each sequence from its own seed). A step
is one chunk-prefill call over this rank's sequences. Under torchrun the 64
sequences are split contiguously over the ranks (64/N each; independent
(sequence, head) pairs, no collective on the data path): strong scaling.
After timing, an untimed NCCL gather brings every rank's outputs to rank 0,
which recomputes the whole batch and checks them bit for bit (gather_check).

  value    Mtok/s over all ranks, inputs resident in HBM (token = one position
           of one sequence across all 16 heads), device-timed with CUDA events,
           max over ranks
  e2e      the same metric through the public API with pinned host buffers:
           H2D of q/k/v/g/beta and D2H of core_attn_out + final_state timed,
           in sub-batches on three streams so copies overlap the kernel
  roofline dominant kernel (chunk_pipe_kernel) against MEASURED_PEAKS.json
  cpu_baseline the reference's own run_deltanet_chunk_rule (oracle/_ref) or
           the oracle port, on a bounded sample, all host threads

--config 0: the chunk rule alone at H16 S104 fp32, latency per call, with the
            reference's chunk rule on one core beside it.
--config 1: the fused decode step (batch 64), CPU restatement beside it.
--config 3/4: full-model prefill / greedy decode (config 4: 256 sequences split
            over the ranks); --exact times the exact-order path.
--impl reference times the reference CPU implementation on the same metric.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, K, V, C = 16, 128, 128, 64


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks + throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, dev):
        self.dev, self.rows, self.proc = dev, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.dev), "--query-gpu=" + self.Q,
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # nvidia-smi's start-up contends with kernel launches: let it
            # print its first sample before the timed region opens
            t_end = time.time() + 5.0
            while not self.rows and time.time() < t_end:
                time.sleep(0.01)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            f = [x.strip() for x in line.split(",")]
            if len(f) == 8:
                self.rows.append(f)

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            self.proc.wait()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        num = lambda x: float(x) if x.replace(".", "").isdigit() else None
        sm = [num(r[1]) for r in self.rows if num(r[1])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[4:]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": num(self.rows[0][2]),
                "reasons": reasons, "samples": len(self.rows)}


def dist_init(args):
    import torch
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import torch.distributed as dist
        backend = "nccl" if args.impl != "reference" else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, device_id=torch.device("cuda", local) if backend == "nccl" else None)
    elif args.impl != "reference":
        torch.cuda.set_device(0)
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, ws):
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda" if dist.get_backend() == "nccl" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- config 2 ---

def make_chunk_inputs(B, S, seed, dev):
    """Seeded on device (bf16 q/k/v with q,k L2-normalised; fp32 g, beta)."""
    import torch
    gen = torch.Generator(device=dev).manual_seed(seed)
    def l2(x):
        return x / torch.sqrt((x * x).sum(-1, keepdim=True) + 1e-6)
    q = l2(torch.randn(B, H, S, K, device=dev, generator=gen)).bfloat16()
    k = l2(torch.randn(B, H, S, K, device=dev, generator=gen)).bfloat16()
    v = torch.randn(B, H, S, V, device=dev, generator=gen).bfloat16()
    g = torch.empty(B, H, S, device=dev).uniform_(-1.0, -0.01, generator=gen)
    b = torch.empty(B, H, S, device=dev).uniform_(0.0, 1.0, generator=gen)
    return q, k, v, g, b


def cpu_reference_sample(threads, S=1024, seqs=None):
    """Times the reference chunk rule (or the oracle port) on a bounded sample;
    returns (Mtok/s, kind, sample description)."""
    import numpy as np
    import oracle
    from tests.golden.gen import chunk_inputs
    seqs = seqs or threads
    q, k, v, g, b = chunk_inputs(H, S, seed=0, batch=seqs)
    out = np.zeros_like(v)
    st = np.zeros((seqs, H, K, V), np.float32)
    ref = oracle.ref_lib()
    import ctypes
    f = ctypes.POINTER(ctypes.c_float)
    P = lambda a: a.ctypes.data_as(f)
    t0 = time.perf_counter()
    if ref is not None:
        rc = ref.ref_chunk_rule_batched(seqs, H, S, K, V, C, P(q), P(k), P(v), P(g), P(b), P(out), P(st), threads)
        kind = "reference"
        assert rc == 0
    else:  # oracle port: one call per sequence, heads over threads
        kind = "port"
        for i in range(seqs):
            oracle.chunk_rule(q[i], k[i], v[i], g[i], b[i], threads=threads)
    dt = time.perf_counter() - t0
    return seqs * S / dt / 1e6, kind, f"{seqs} sequences x {H} heads x {S} tokens, fp32, {threads} threads, {dt:.1f} s"


def shard(total, ws, rank):
    """Contiguous split of `total` independent sequences over ws ranks:
    (first sequence, count) of this rank. Every sequence is owned once."""
    base, extra = divmod(total, ws)
    first = rank * base + min(rank, extra)
    return first, base + (1 if rank < extra else 0)


def shard_inputs(first, count, S, dev):
    """Inputs of sequences [first, first+count): each sequence is drawn from
    its own seed, so a shard is the same whichever rank computes it."""
    import torch
    parts = [make_chunk_inputs(1, S, 1234 + i, dev) for i in range(first, first + count)]
    return tuple(torch.cat([p[j] for p in parts]) for j in range(5))


def bench_chunk(args, ws, rank, local):
    import torch
    import spock_b200
    dev = torch.device("cuda", local)
    S = args.seq
    if args.scaling == "strong":  # 64 sequences sharded over the ranks
        first, B = shard(args.batch, ws, rank)
    else:
        first, B = rank * args.batch, args.batch
    q, k, v, g, b = shard_inputs(first, B, S, dev)
    out = torch.empty(B, H, S, V, dtype=torch.bfloat16, device=dev)
    st = torch.empty(B, H, K, V, dtype=torch.float32, device=dev)
    ctx = spock_b200.Context.get(local)
    stream = torch.cuda.current_stream()
    run = lambda: spock_b200.chunk_prefill(q, k, v, g, b, out_dtype=torch.bfloat16, out=out,
                                           final_state=st, ctx=ctx, stream=stream)
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    ctx.sync()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    n0 = spock_b200.lib().spock_kernel_launch_count()
    barrier(ws)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for e0, e1 in evs:
            e0.record(stream)
            run()
            e1.record(stream)
        t1.record(stream)
        torch.cuda.synchronize()
    barrier(ws)
    launches = spock_b200.lib().spock_kernel_launch_count() - n0
    ctx.sync()
    total_ms = max_over_ranks(t0.elapsed_time(t1), ws)
    kern_ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs)
    kern_ms = max_over_ranks(kern_ms, ws)
    ms_step = total_ms / args.steps
    tokens_step = (args.batch if args.scaling == "strong" else B * ws) * S
    value = tokens_step / (ms_step / 1e3) / 1e6

    # untimed: gather every rank's outputs to rank 0 over NCCL and check them
    # bit for bit against rank 0 recomputing the whole batch (the kernel is
    # deterministic, so a correct shard/gather reproduces it exactly)
    gather_ok = None
    if ws > 1 and args.gather and args.scaling == "strong":
        gather_ok = gather_check(args, ws, rank, dev, out, st, ctx)

    # end to end through the public API with pinned host buffers: the batch
    # goes through in sub-batches on three streams, so the H2D copy of one
    # sub-batch, the kernel of the previous one and the D2H copy of the one
    # before overlap (separate copy engines per direction)
    hq = [x.cpu().pin_memory() for x in (q, k, v, g, b)]
    hout = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    hst = torch.empty(st.shape, dtype=st.dtype).pin_memory()
    dq = [torch.empty_like(x) for x in (q, k, v, g, b)]
    h2d = sum(x.numel() * x.element_size() for x in hq)
    d2h = hout.numel() * hout.element_size() + hst.numel() * hst.element_size()
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    sub = max(1, min(B, args.e2e_sub))
    cuts = [B * i // sub for i in range(sub + 1)]
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)

    def e2e_step():
        ev_prev = torch.cuda.Event()
        ev_prev.record(stream)
        s_in.wait_event(ev_prev)  # the previous step's kernels are done with the inputs
        for c0, c1 in zip(cuts[:-1], cuts[1:]):
            if c0 == c1:
                continue
            with torch.cuda.stream(s_in):
                for d_, h_ in zip(dq, hq):
                    d_[c0:c1].copy_(h_[c0:c1], non_blocking=True)
                e_in = torch.cuda.Event()
                e_in.record(s_in)
            stream.wait_event(e_in)
            spock_b200.chunk_prefill(*(d_[c0:c1] for d_ in dq), out_dtype=torch.bfloat16, out=out[c0:c1],
                                     final_state=st[c0:c1], ctx=ctx, stream=stream)
            e_c = torch.cuda.Event()
            e_c.record(stream)
            s_out.wait_event(e_c)
            with torch.cuda.stream(s_out):
                hout[c0:c1].copy_(out[c0:c1], non_blocking=True)
                hst[c0:c1].copy_(st[c0:c1], non_blocking=True)
        e_done = torch.cuda.Event()
        e_done.record(s_out)
        stream.wait_event(e_done)
    e2e_step()
    torch.cuda.synchronize()
    barrier(ws)
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    a1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(a0.elapsed_time(a1), ws) / e2e_steps
    e2e_val = tokens_step / (e2e_ms / 1e3) / 1e6

    hbm, tf, pk = peaks()
    alg_bytes = B * H * S * (3 * K * 2 + 8 + V * 2) + B * H * K * V * 4
    alg_flops = B * H * S * 2 * (5 * C * K + 3 * K * V)
    achieved_gbs = alg_bytes / (kern_ms / 1e3) / 1e9
    achieved_tf = alg_flops / (kern_ms / 1e3) / 1e12
    t_hbm, t_tc = alg_bytes / (hbm * 1e9), alg_flops / (tf * 1e12)
    res = {
        "metric": "chunk-prefill Mtok/s (token = one sequence position across all 16 heads)",
        "value": round(value, 3), "unit": "Mtok/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
        "dtype": "bf16 in/out, fp16 tensor-core operands, fp32 state+accumulation", "data": "synthetic (seeded, config-0 distributions)",
        "config": {"workload": "config 2: batched chunk prefill", "sequences": args.batch if args.scaling == "strong" else B * ws,
                   "sequences_per_gpu": B, "heads": H,
                   "seq_len": S, "chunk": C, "k_dim": K, "v_dim": V,
                   "parallelism": f"dp{ws} over sequences ({args.scaling} scaling)",
                   "l2": "inputs (%.1f GB/GPU) larger than L2" % (alg_bytes / 1e9)},
        "per_gpu_Mtok_s": round(value / ws, 3),
        **({"gather_check": gather_ok} if gather_ok is not None else {}),
        "e2e": {"value": round(e2e_val, 4), "unit": "Mtok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms, 3), "sub_batches": sub},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm" if t_hbm >= t_tc else "tensor", "achieved": round(achieved_gbs, 1),
                     "peak": hbm, "unit": "GB/s", "frac": round(achieved_gbs / hbm, 4),
                     # DRAM read + write per launch from one ncu capture (160 pairs x 8192 tokens:
                     # 1.337 GB), scaled by token-heads to this launch
                     "traffic": int(1.337e9 / (160 * 8192) * B * 16 * S), "traffic_source": "ncu, scaled",
                     "peak_source": pk,
                     "tensor": {"achieved": round(achieved_tf, 1), "peak": tf, "unit": "TFLOP/s",
                                "frac": round(achieved_tf / tf, 4)},
                     "kernel_ms": round(kern_ms, 4), "alg_bytes": alg_bytes, "alg_flops": alg_flops},
        "clocks": clk.summary(),
    }
    return res


def gather_check(args, ws, rank, dev, out, st, ctx):
    """NCCL gather of every rank's core_attn_out and final state to rank 0, then
    rank 0 recomputes each shard and compares bit for bit. Returns the verdict
    on every rank (broadcast)."""
    import torch
    import torch.distributed as dist
    import spock_b200
    shapes = [shard(args.batch, ws, r) for r in range(ws)]
    ok = True
    if rank == 0:
        bufs_o = [torch.empty((n,) + tuple(out.shape[1:]), dtype=out.dtype, device=dev) for _, n in shapes]
        bufs_s = [torch.empty((n,) + tuple(st.shape[1:]), dtype=st.dtype, device=dev) for _, n in shapes]
    else:
        bufs_o = bufs_s = None
    # gather of unequal shards: one point-to-point pair per rank (NCCL over NVLink)
    for r in range(1, ws):
        if rank == r:
            dist.send(out, 0)
            dist.send(st, 0)
        elif rank == 0:
            dist.recv(bufs_o[r], r)
            dist.recv(bufs_s[r], r)
    if rank == 0:
        bufs_o[0].copy_(out)
        bufs_s[0].copy_(st)
        for (first, n), go, gs in zip(shapes, bufs_o, bufs_s):
            q, k, v, g, b = shard_inputs(first, n, args.seq, dev)
            ro, rs = spock_b200.chunk_prefill(q, k, v, g, b, out_dtype=torch.bfloat16, ctx=ctx)
            torch.cuda.synchronize()
            ok = ok and torch.equal(ro, go) and torch.equal(rs, gs)
            del q, k, v, g, b, ro, rs
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.broadcast(flag, 0)
    return bool(flag.item())


# ---------------------------------------------------------------- config 1 ---

def bench_decode(args, ws, rank, local):
    import numpy as np
    import torch
    import spock_b200
    from tests.golden.gen import decode_inputs
    dev = torch.device("cuda", local)
    B = args.batch
    layers = args.layers  # independent layer states so successive steps stream fresh HBM
    d = decode_inputs(B, seed=rank)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    h16 = lambda a: T(a.view(np.int16))
    layer = spock_b200.DeltaNetLayer(h16(d["conv_w"]), T(d["a_log_bias"]), T(d["norm_w"]))
    states = [T(d["state"]) for _ in range(layers)]
    convs = [h16(d["conv_state"]) for _ in range(layers)]
    qkv0 = h16(d["qkv"])
    qkv = [qkv0.clone() for _ in range(layers)]
    a, b_, z = h16(d["a"]), h16(d["b"]), h16(d["z"])
    out = torch.empty((B, 2048), dtype=torch.int16, device=dev)
    ctx = spock_b200.Context.get(local)
    stream = torch.cuda.current_stream()

    def step():
        for l in range(layers):
            spock_b200.deltanet_decode_step(layer, qkv[l], convs[l], states[l], a, b_, z, out=out, ctx=ctx, stream=stream)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # The step's launches are captured once into a CUDA graph (as the model
    # session does), so a small batch measures the kernels, not the Python
    # and ctypes cost of issuing them.
    graph = torch.cuda.CUDAGraph()
    n0 = spock_b200.lib().spock_kernel_launch_count()
    with torch.cuda.graph(graph, capture_error_mode="relaxed"):
        stream = torch.cuda.current_stream()
        step()
    per_step = spock_b200.lib().spock_kernel_launch_count() - n0
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier(ws)
    with ClockSampler(local) as clk:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        t1.record(stream)
        torch.cuda.synchronize()
    launches = per_step * args.steps
    ms = max_over_ranks(t0.elapsed_time(t1), ws) / args.steps
    per_launch_ms = ms / layers
    value = B * layers * ws / (ms / 1e3)  # sequence-layer steps per second
    hbm, tf, pk = peaks()
    alg = B * (H * K * V * 4 * 2 + 6144 * 4 * 2 * 2 + 6144 * 2 + 2048 * 2 * 2 + 64) + 6144 * 8 + 512 + 128
    gbs = alg / (per_launch_ms / 1e3) / 1e9
    return {
        "metric": "fused DeltaNet decode step: sequence-layer steps/s", "value": round(value, 1), "unit": "steps/s",
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16 io, fp32 state",
        "data": "synthetic (seeded, config-1 distributions)",
        "config": {"workload": "config 1: fused decode step", "batch": B, "layers_per_step": layers,
                   "l2": "%d independent layer states (%.0f MB) larger than L2" % (layers, layers * B * 1.05)},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                     # DRAM read + write of one launch from an ncu capture at batch 64 (71.4 + 13.1 MB;
                     # part of the written state is still in L2 when the launch ends), scaled by batch
                     "frac": round(gbs / hbm, 4), "traffic": int(84.5e6 * B / 64), "traffic_source": "ncu, scaled",
                     "peak_source": pk,
                     "kernel_us": round(per_launch_ms * 1e3, 2), "alg_bytes": alg},
        "clocks": clk.summary(),
    }


# ------------------------------------------------------------ configs 3 / 4 ---

def model_weights_gpu(layers, vocab, seed, dev):
    """Random-init Qwen3.5-0.8B-layout weights (config 3 distributions), drawn on
    the GPU for speed and returned as host arrays for spock_model_set_weight."""
    import numpy as np
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    def mat(o, i, sd=0.02):
        return (torch.randn(o, i, device=dev, generator=g) * sd).half().view(torch.int16).cpu().numpy().view(np.uint16)
    def vec16(n, sd=0.1):
        return (torch.randn(n, device=dev, generator=g) * sd).half().view(torch.int16).cpu().numpy().view(np.uint16)
    w = {"embedding": mat(vocab, 1024), "final_norm": vec16(1024)}
    for i in range(layers):
        p = f"layer.{i}."
        w[p + "input_norm"] = vec16(1024)
        w[p + "post_norm"] = vec16(1024)
        w[p + "mlp_gate"] = mat(3584, 1024)
        w[p + "mlp_up"] = mat(3584, 1024)
        w[p + "mlp_down"] = mat(1024, 3584)
        if i % 4 == 3:
            w[p + "attn_q"] = mat(4096, 1024)
            w[p + "attn_k"] = mat(512, 1024)
            w[p + "attn_v"] = mat(512, 1024)
            w[p + "attn_q_norm"] = vec16(256)
            w[p + "attn_k_norm"] = vec16(256)
            w[p + "attn_o"] = mat(1024, 2048)
        else:
            w[p + "delta_in_proj_qkv"] = mat(6144, 1024)
            w[p + "delta_in_proj_z"] = mat(2048, 1024)
            w[p + "delta_in_proj_a"] = mat(16, 1024)
            w[p + "delta_in_proj_b"] = mat(16, 1024)
            w[p + "delta_conv"] = mat(6144, 4)
            w[p + "delta_norm"] = (1.0 + 0.1 * torch.randn(128, device=dev, generator=g)).float().cpu().numpy()
            w[p + "delta_a_log"] = (torch.rand(16, device=dev, generator=g) * 3 - 2).float().cpu().numpy()
            w[p + "delta_dt_bias"] = vec16(16)
            w[p + "delta_out_proj"] = mat(1024, 2048)
    return w


def bench_model(args, ws, rank, local):
    """Config 4 (greedy decode after a 512-token prompt) or config 3 (prompt
    prefill). A step is one token for every sequence of this GPU's batch."""
    import numpy as np
    import torch
    import spock_b200
    dev = torch.device("cuda", local)
    P, layers, vocab = args.prompt, 24, 248320
    B = shard(args.batch, ws, rank)[1] if args.scaling == "strong" else args.batch
    total_seqs = args.batch if args.scaling == "strong" else B * ws
    w = model_weights_gpu(layers, vocab, 7, dev)
    m = spock_b200.Model(layers, vocab, max_batch=B, max_seq=P + args.steps + args.warmup + 48, device=local,
                         exact=args.exact)
    m.set_weights(w)
    cpu_base = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu_base = cpu_model_sample(w, layers, vocab)
    del w
    m.reset(B)
    stream = torch.cuda.Stream(device=dev)
    prompt = torch.randint(0, vocab, (B, P), generator=torch.Generator().manual_seed(rank), dtype=torch.int32).to(dev)
    cnt = spock_b200.lib().spock_kernel_launch_count
    with torch.cuda.stream(stream):
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0 = cnt()
        m.generate(prompt[:, :1].contiguous(), 1, stream=stream)  # captures the step graph: counts its kernels once
        per_step = cnt() - c0
        m.reset(B)
        stream.synchronize()
        if args.config == 3:
            # layer-major prefill of the P-token prompt (spock_model_prefill, via generate's
            # first token), timed as a whole
            for i in range(max(3, args.warmup)):
                m.reset(B)
                c0 = cnt()
                m.generate(prompt, 1, stream=stream)  # warm-up: scratch, eager run, graph capture
                if i == 0:
                    per_pf = cnt() - c0  # the eager run counts every kernel of one prefill
            # each timed prefill between its own events (the session reset
            # between prefills is outside them)
            n_pf = max(1, args.steps)
            evp = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_pf)]
            barrier(ws)
            with ClockSampler(local) as clk:
                for e0, e1 in evp:
                    m.reset(B)
                    e0.record(stream)
                    m.generate(prompt, 1, stream=stream)
                    e1.record(stream)
                stream.synchronize()
            steps = P
        else:
            m.generate(prompt, 1 + args.warmup, stream=stream)  # prefill + graph capture + warm-up
            stream.synchronize()
            tok = torch.zeros(B, dtype=torch.int32, device=dev)
            barrier(ws)
            with ClockSampler(local) as clk:
                t0.record(stream)
                for _ in range(args.steps):
                    tok, _h = m.step(tok, stream=stream)
                t1.record(stream)
                stream.synchronize()
            steps = args.steps
    if args.config == 3:
        launches = per_pf * n_pf
        ms = max_over_ranks(statistics.mean(e0.elapsed_time(e1) for e0, e1 in evp), ws) / steps
    else:
        launches = per_step * steps  # graph replays: kernels per step x timed steps
        ms = max_over_ranks(t0.elapsed_time(t1), ws) / steps
    value = total_seqs / (ms / 1e3)
    hbm, tf, pk = peaks()
    w_bytes = 752.4e6 * 2
    state_bytes = B * 18 * (16 * 128 * 128 * 4 * 2 + 6144 * 4 * 2 * 2)
    kv_bytes = B * 6 * 2 * 2 * 256 * 2 * (P + steps // 2)
    alg = w_bytes + state_bytes + kv_bytes
    gbs = alg / (ms / 1e3) / 1e9
    if args.config == 3:
        # prefill is tensor-bound: linear layers (498.1 M params) over every token, the chunk rule
        # (180 224 FLOP per token-head, 18 layers x 16 heads), causal attention (6 layers, 8 heads,
        # QK and PV over head 256) and the LM head for each sequence's last token
        flops = B * (2 * 498.1e6 * P + 18 * 16 * P * 180224.0 + 6 * 8 * 4 * 256 * P * (P + 1) / 2 + 2 * 254.3e6)
        roof = {"bound": "tensor", "achieved": round(flops / (ms * steps / 1e3) / 1e12, 2), "peak": tf,
                "unit": "TFLOP/s", "frac": round(flops / (ms * steps / 1e3) / 1e12 / tf, 4), "traffic": None,
                "peak_source": pk, "alg_flops": flops}
    else:
        roof = {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s", "frac": round(gbs / hbm, 4),
                "traffic": None, "peak_source": pk, "alg_bytes_per_step": int(alg)}
    # end to end through the public API: host prompt -> device, generate, tokens -> host
    hp = prompt[:, : min(P, 16)].contiguous().cpu().pin_memory()
    n_e2e = 16
    m.reset(B)
    with torch.cuda.stream(stream):
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        dp = hp.to(dev, non_blocking=True)
        out = m.generate(dp, n_e2e, stream=stream)
        ho = out.to("cpu", non_blocking=True)
        a1.record(stream)
        stream.synchronize()
    e2e_ms = max_over_ranks(a0.elapsed_time(a1), ws)
    e2e_val = total_seqs * (hp.shape[1] + n_e2e - 1) / (e2e_ms / 1e3)
    m.close()
    name = "full-model greedy decode tok/s" if args.config == 4 else "full-model layer-major prefill tok/s"
    res = {
        "metric": name, "value": round(value, 1), "unit": "tok/s", "n_gpus": ws, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "fp16 weights/activations, fp32 accumulation and DeltaNet state",
        "data": "synthetic (random-init Qwen3.5-0.8B layout, seeded random prompt)",
        "config": {"workload": f"config {args.config}", "sequences": total_seqs, "sequences_per_gpu": B, "prompt": P,
                   "layers": layers, "path": "exact order (bit-identical tokens)" if args.exact else
                   "tensor-core projections + chunk-rule prefill",
                   "vocab": vocab, "parallelism": f"dp{ws} over sequences ({args.scaling} scaling)",
                   "l2": "weights (1.5 GB) larger than L2",
                   **({"prefills_timed": n_pf, "step": "one prompt token (ms_per_step = prefill ms / prompt)"}
                      if args.config == 3 else {})},
        "e2e": {"value": round(e2e_val, 1), "unit": "tok/s", "h2d_bytes_per_step": int(hp.numel() * 4 / (hp.shape[1] + n_e2e - 1)),
                "d2h_bytes_per_step": int(B * 4), "note": f"{hp.shape[1]}-token prompt + {n_e2e} new tokens via spock_model_generate"},
        "gpu_launches": int(launches),
        "roofline": roof,
        "clocks": clk.summary(),
    }
    if cpu_base:
        res["cpu_baseline"] = cpu_base
    return res


def cpu_model_sample(w, layers, vocab):
    """The CPU restatement of the decode path (oracle/model.cpp, the reference
    has no CPU decode of its own) on a bounded sample: greedy decode steps of
    one sequence, all host threads and one. tok/s; one step = one token."""
    import numpy as np
    import oracle
    threads = os.cpu_count() or 1
    cpu = oracle.Model(w, layers, vocab, 16)
    rates = {}
    for th, n in ((threads, 6), (1, 2)):
        cpu.reset(1)
        cpu.step(np.array([1], np.int32), threads=th)
        t0 = time.perf_counter()
        for i in range(n):
            cpu.step(np.array([i + 2], np.int32), threads=th)
        rates[th] = n / (time.perf_counter() - t0)
    return {"value": round(rates[threads], 3), "unit": "tok/s", "cores": threads, "kind": "port",
            "single_core_value": round(rates[1], 3),
            "sample": f"greedy decode steps of 1 sequence ({layers} layers, vocab {vocab}): 6 steps on {threads} "
                      "threads, 2 on 1 thread (token-serial: the restatement's prefill rate is the same per token)"}


def cpu_decode_sample(B):
    """Oracle restatement of the fused decode step (conv_l2_qk + recurrent
    gbeta norm gate) at batch B: sequence-layer steps/s on all threads and one."""
    import numpy as np
    import oracle
    from tests.golden.gen import decode_inputs
    threads = os.cpu_count() or 1
    d = decode_inputs(B, seed=0)
    rates = {}
    for th, reps in ((threads, 5), (1, 2)):
        t0 = time.perf_counter()
        for _ in range(reps):
            qkv, _ = oracle.conv_l2_qk(d["qkv"], d["conv_state"], d["conv_w"], threads=th)
            oracle.rec_norm_gate(qkv, d["state"], d["a"], d["b"], d["a_log_bias"], d["z"], d["norm_w"], threads=th)
        rates[th] = B * reps / (time.perf_counter() - t0)
    return {"value": round(rates[threads], 1), "unit": "steps/s", "cores": threads, "kind": "port",
            "single_core_value": round(rates[1], 1),
            "sample": f"batch {B}, one layer: 5 steps on {threads} threads, 2 on 1 thread"}


# ---------------------------------------------------------------- config 0 ---

def bench_config0(args, ws, rank, local):
    """the chunk rule alone, H16, S104 (padded to 128), C64,
    fp32, one call. Latency per call with L2 flushed between calls; the
    reference's own run_deltanet_chunk_rule on one core beside it."""
    import numpy as np
    import torch
    import spock_b200
    import oracle
    from tests.golden.gen import chunk_inputs
    dev = torch.device("cuda", local)
    q, k, v, g, b = chunk_inputs(16, 104, seed=0, batch=1)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    dq, dk, dv, dg, db = map(T, (q, k, v, g, b))
    out = torch.empty((1, 16, 104, 128), device=dev)
    st = torch.empty((1, 16, 128, 128), device=dev)
    ctx = spock_b200.Context.get(local)
    stream = torch.cuda.current_stream()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > L2 (126 MB)
    run = lambda: spock_b200.chunk_prefill(dq, dk, dv, dg, db, out_dtype=torch.float32, out=out, final_state=st,
                                           ctx=ctx, stream=stream)
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    n0 = spock_b200.lib().spock_kernel_launch_count()
    with ClockSampler(local) as clk:
        for e0, e1 in evs:
            flush.zero_()
            e0.record(stream)
            run()
            e1.record(stream)
        torch.cuda.synchronize()
    launches = spock_b200.lib().spock_kernel_launch_count() - n0 - 0
    ctx.sync()
    us = statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs) * 1e3
    # e2e: host fp32 buffers in, outputs back, through the public API
    hin = [torch.from_numpy(np.ascontiguousarray(a)).pin_memory() for a in (q, k, v, g, b)]
    hout = torch.empty(out.shape).pin_memory()
    hst = torch.empty(st.shape).pin_memory()
    e2e = []
    for _ in range(args.steps):
        flush.zero_()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for d_, h_ in zip((dq, dk, dv, dg, db), hin):
            d_.copy_(h_, non_blocking=True)
        run()
        hout.copy_(out, non_blocking=True)
        hst.copy_(st, non_blocking=True)
        a1.record(stream)
        torch.cuda.synchronize()
        e2e.append(a0.elapsed_time(a1) * 1e3)
    h2d = sum(x.numel() * 4 for x in hin)
    d2h = (hout.numel() + hst.numel()) * 4
    # the reference's own chunk rule (oracle/_ref) on one core, same inputs
    ref = oracle.ref_lib()
    kind = "reference" if ref is not None else "port"
    t0 = time.perf_counter()
    reps = 5
    for _ in range(reps):
        oracle.chunk_rule(q[0], k[0], v[0], g[0], b[0], use_reference=ref is not None, threads=1)
    cpu_us = (time.perf_counter() - t0) / reps * 1e6
    hbm, tf, pk = peaks()
    alg = 3 * 16 * 104 * 128 * 4 + 2 * 16 * 104 * 4 + 16 * 104 * 128 * 4 + 16 * 128 * 128 * 4
    return {
        "metric": "config-0 chunk rule latency per call (H16 S104 C64 fp32)", "value": round(us, 2), "unit": "us",
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 5),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32 in/out, fp16 hi/lo tensor-core "
        "operands, fp32 state+accumulation", "data": "synthetic (seeded, config-0 distributions)",
        "config": {"workload": "config 0: chunk rule alone", "heads": 16, "seq_len": 104, "chunk": 64, "k_dim": 128,
                   "v_dim": 128, "l2": "256 MB buffer written between timed calls"},
        "e2e": {"value": round(statistics.mean(e2e), 2), "unit": "us", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "achieved": round(alg / (us / 1e6) / 1e9, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(alg / (us / 1e6) / 1e9 / hbm, 4), "traffic": None, "peak_source": pk,
                     "note": "latency-bound: 16 (head) CTAs, 2 serial chunks each"},
        "cpu_baseline": {"value": round(cpu_us, 1), "unit": "us", "cores": 1, "kind": kind,
                         "sample": "the whole config-0 call, 5 repetitions, 1 thread"},
        "clocks": clk.summary(),
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="spock_b200", choices=["spock_b200", "reference"])
    ap.add_argument("--config", type=int, default=2, choices=[0, 1, 2, 3, 4])
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--seq", type=int, default=8192)
    ap.add_argument("--layers", type=int, default=18)
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--e2e-sub", type=int, default=8, help="config 2 e2e: sub-batches overlapped on 3 streams")
    ap.add_argument("--scaling", default=None, choices=["strong", "weak"],
                    help="strong: --batch sequences in total, split over the ranks (config 2 and 4 default); "
                         "weak: --batch sequences per rank")
    ap.add_argument("--no-gather", dest="gather", action="store_false",
                    help="config 2, N > 1: skip the untimed NCCL gather + check of the outputs")
    ap.add_argument("--exact", action="store_true", help="configs 3/4: the exact-order model path")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.batch is None:
        args.batch = {0: 1, 1: 64, 2: 64, 3: 1, 4: 256}[args.config]
    if args.scaling is None:
        args.scaling = "strong" if args.config in (2, 4) else "weak"
    args.warmup = max(args.warmup, 3) if args.impl != "reference" else args.warmup
    ws, rank, local = dist_init(args)

    if args.impl == "reference":
        if rank == 0:
            threads = os.cpu_count() or 1
            vals, kind, sample = [], None, None
            for i in range(args.warmup + args.steps):
                v, kind, sample = cpu_reference_sample(threads, S=512)
                if i >= args.warmup:
                    vals.append(v)
            val = statistics.mean(vals)
            print(json.dumps({
                "impl": "reference", "metric": "chunk-prefill Mtok/s (token = one sequence position across all 16 heads)",
                "value": round(val, 6), "unit": "Mtok/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
                "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded, config-0 distributions)",
                "config": {"workload": "config 2: batched chunk prefill (bounded sample per step)", "heads": H,
                           "chunk": C, "k_dim": K, "v_dim": V},
                "cpu_baseline": {"value": round(val, 6), "unit": "Mtok/s", "cores": threads, "kind": kind, "sample": sample},
                "e2e": {"value": round(val, 6), "unit": "Mtok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
                flush=True)
        return

    if args.config == 2:
        res = bench_chunk(args, ws, rank, local)
    elif args.config == 0:
        res = bench_config0(args, ws, rank, local)
    elif args.config == 1:
        res = bench_decode(args, ws, rank, local)
        if rank == 0 and ws == 1 and not args.no_cpu_baseline:
            res["cpu_baseline"] = cpu_decode_sample(args.batch)
    else:
        res = bench_model(args, ws, rank, local)
    if rank == 0:
        if ws == 1 and not args.no_cpu_baseline and args.config == 2:
            threads = os.cpu_count() or 1
            v, kind, sample = cpu_reference_sample(threads, S=1024)
            res["cpu_baseline"] = {"value": round(v, 6), "unit": "Mtok/s", "cores": threads, "kind": kind, "sample": sample}
        print(json.dumps(res), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
