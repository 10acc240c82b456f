"""Shared checks. The parity metric is the reference probes' own:
max |gpu - ref| / max(1, |ref|) (apps/spock-deltanet-chunk-prefill-probe.cpp:440-444)."""
import numpy as np


def max_rel(a, ref):
    a = np.asarray(a, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(a - ref) / np.maximum(1.0, np.abs(ref)))) if a.size else 0.0


def fp16_ulp_diff(a_bits, b_bits):
    """Distance in representable fp16 values; opposite signs count as huge
    (the reference's ULP policy never passes a sign flip)."""
    a = np.asarray(a_bits, np.uint16).astype(np.int32)
    b = np.asarray(b_bits, np.uint16).astype(np.int32)
    def ordered(x):
        mag = x & 0x7FFF
        return np.where(x & 0x8000, -mag, mag)
    d = np.abs(ordered(a) - ordered(b))
    sign_flip = ((a ^ b) & 0x8000).astype(bool) & ((a & 0x7FFF) != 0) & ((b & 0x7FFF) != 0)
    return np.where(sign_flip, 1 << 16, d)


def close16(a_bits, b_bits, ulp=2, abs_tol=2.0 ** -10):
    """fp16 values (given as uint16 bits) agree within `ulp` ulps, or within
    abs_tol absolutely (outputs are O(1); near zero a tiny absolute difference
    spans many ulps)."""
    a = np.asarray(a_bits, np.uint16).view(np.float16).astype(np.float64)
    b = np.asarray(b_bits, np.uint16).view(np.float16).astype(np.float64)
    return bool(np.all((fp16_ulp_diff(a_bits, b_bits) <= ulp) | (np.abs(a - b) <= abs_tol)))
