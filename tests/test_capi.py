"""The C-ABI library builds, loads and exports every symbol its header declares;
host-side validation behaves like the reference's (no GPU needed)."""
import ctypes
import os
import re

import pytest

import spock_b200

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    txt = open(os.path.join(ROOT, "include", "spock_b200.h")).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*|uint64_t)\s+(spock_\w+)\s*\(", txt, re.M)))


def test_header_declares_the_python_export_list():
    assert declared_symbols() == sorted(spock_b200.EXPORTED)


def test_library_exports_every_declared_symbol():
    L = spock_b200.lib()
    for name in declared_symbols():
        assert hasattr(L, name), name


def test_null_context_is_rejected_without_gpu():
    L = spock_b200.lib()
    d = spock_b200.ChunkDesc(1, 1, 1, 128, 128, 64, 0, 0, 0, 0)
    rc = L.spock_chunk_prefill(None, ctypes.byref(d), *([None] * 9))
    assert rc == spock_b200.SPOCK_ERR_INVALID
    assert b"ctx is NULL" in L.spock_last_error(None)


def test_create_reports_error_text_instead_of_crashing():
    import torch
    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    h = ctypes.c_void_p()
    rc = spock_b200.lib().spock_create(0, ctypes.byref(h))
    assert rc != spock_b200.SPOCK_OK and h.value is None
    assert spock_b200.lib().spock_last_error(None)


@pytest.mark.parametrize("field", ["num_heads", "sequence_length", "key_dim", "value_dim", "chunk_size"])
def test_run_chunk_rule_rejects_zero_fields(field):
    cfg = spock_b200.DeltaNetChunkConfig(2, 5, 128, 128, 64)
    setattr(cfg, field, 0)
    with pytest.raises(spock_b200.SpockError, match="must be non-zero"):
        spock_b200.run_deltanet_chunk_rule(cfg, spock_b200.DeltaNetChunkInputs())


def test_run_chunk_rule_rejects_size_mismatch():
    cfg = spock_b200.DeltaNetChunkConfig(1, 2, 128, 128, 64)
    with pytest.raises(spock_b200.SpockError, match="query size mismatch"):
        spock_b200.run_deltanet_chunk_rule(cfg, spock_b200.DeltaNetChunkInputs(query=[0.0] * 3))
