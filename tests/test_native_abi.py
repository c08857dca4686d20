"""The C-ABI library loads, exports every entry point the header declares, and
rejects bad arguments on the host (no GPU needed)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from tilequant_b200 import _native as N

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "tilequant_b200.h"


def _declared():
    text = HEADER.read_text()
    return re.findall(r"^TQ_API\s+(?:const\s+)?\w+\**\s+(tq_\w+)\s*\(", text, flags=re.M)


@pytest.fixture(scope="module")
def lib():
    if not N.LIB_PATH.exists():
        from tilequant_b200 import build

        build.build()
    return N.load()


def test_header_declares_entry_points():
    names = _declared()
    assert len(names) >= 14
    assert set(names) == set(N.SIGNATURES), "ctypes table and header disagree"


def test_every_declared_symbol_is_exported(lib):
    for name in _declared():
        assert hasattr(lib, name), name


def test_abi_version_and_status_strings(lib):
    assert lib.tq_abi_version() == N.ABI_VERSION
    assert lib.tq_status_string(N.TQ_ERR_INVALID) == b"TQ_ERR_INVALID"
    assert lib.tq_status_string(N.TQ_ERR_TIMEOUT) == b"TQ_ERR_TIMEOUT"


def test_host_side_argument_checks(lib):
    # bad dtype / shapes are rejected before any CUDA call
    assert lib.tq_act_scales(None, 7, 4, 64, 64, 1, None, None) == N.TQ_ERR_INVALID
    assert b"dtype" in lib.tq_last_error()
    assert lib.tq_quantize_act(None, 0, -1, 64, 64, 1, None, 64, None, None) == N.TQ_ERR_INVALID
    # tile grid that does not match (m, k)
    rc = lib.tq_gemm_mixed(None, 64, None, None, None, None, None, 0, None, 64, None, None, None, 0, 0, None, 64,
                           0, None, 1, 64, 64, 2, 1, 0, 0, None, None)
    assert rc == N.TQ_ERR_INVALID and b"tile grid" in lib.tq_last_error()
    # tile counts that do not cover the grid
    rc = lib.tq_gemm_mixed(None, 64, None, None, None, None, None, 3, None, 64, None, None, None, 0, 0, None, 64,
                           0, None, 1, 64, 64, 1, 1, 0, 0, None, None)
    assert rc == N.TQ_ERR_INVALID
    # split_k beyond 16
    dummy = ctypes.c_void_p(16)
    rc = lib.tq_gemm_mixed(dummy, 64, dummy, dummy, dummy, dummy, dummy, 1, None, 64, None, None, None, 0, 0, dummy, 64,
                           0, None, 1, 64, 64, 1, 1, 17, 0, None, None)
    assert rc == N.TQ_ERR_INVALID and b"split_k" in lib.tq_last_error()
    # fused decode form is limited to 64 rows
    rc = lib.tq_gemm_mixed_fused_quant(dummy, 64, 0, dummy, dummy, dummy, dummy, 1, None, None, None, 0, dummy, 64, 0,
                                       None, 65, 64, 64, 1, 1, 0, None, None)
    assert rc == N.TQ_ERR_INVALID
    assert lib.tq_calib_iaa_tile_scores(dummy, 0, 64, 64, 64, dummy, 0, dummy, dummy, None) == N.TQ_ERR_INVALID


def test_peer_sum_host_side_checks(lib):
    # exchange layout: 16-byte words {v, call, v, call} [2][world][slots][128]
    assert lib.tq_peer_buffer_bytes(2, 1024) == 2 * 2 * 1024 * 128 * 16
    assert lib.tq_peer_buffer_bytes(3, 5) == 2 * 3 * 5 * 128 * 16
    assert lib.tq_peer_buffer_bytes(0, 16) == 0 and lib.tq_peer_buffer_bytes(9, 16) == 0
    assert lib.tq_peer_buffer_bytes(2, 0) == 0 and lib.tq_peer_buffer_bytes(2, 65537) == 0
    out = ctypes.c_void_p()
    assert lib.tq_peer_alloc(0, 16, ctypes.byref(out)) == N.TQ_ERR_INVALID and out.value is None
    assert lib.tq_peer_reset(None, 2, 16, None, None) == N.TQ_ERR_INVALID
    dummy = ctypes.c_void_p(16)
    args = [dummy, 64, dummy, dummy, dummy, dummy, dummy, 1, None, 64, None, None, None, 0, 0, dummy, 64, 0, None,
            1, 64, 64, 1, 1, 0]
    for world, rank, slots, timeout in [(9, 0, 16, 10**9), (2, 2, 16, 10**9), (2, 0, 0, 10**9), (2, 0, 16, 0)]:
        rc = lib.tq_gemm_mixed_peer_sum(*args, dummy, dummy, world, rank, slots, timeout, None, None)
        assert rc == N.TQ_ERR_INVALID, (world, rank, slots, timeout)
    rc = lib.tq_gemm_mixed_peer_sum(*args, None, dummy, 2, 0, 16, 10**9, None, None)
    assert rc == N.TQ_ERR_INVALID and b"exchange" in lib.tq_last_error()


def test_python_errors_map_to_reference_exceptions(lib):
    with pytest.raises(ValueError):
        N.check(N.TQ_ERR_INVALID, "x")
    with pytest.raises(N.TileQuantError):
        N.check(N.TQ_ERR_CUDA, "x")


def test_integration_binding_matches_the_library():
    """The ctypes binding shown to maintainers names every
    entry point of the header and gives each the argument count and types this
    package's own binding uses."""
    doc = (ROOT / "INTEGRATION.md").read_text()
    start = doc.index("```python", doc.index("## 2."))
    block = doc[start:doc.index("```", start + 10)]
    block = re.sub(r"\[\s*([^\]]*?)\]", lambda m: "[" + " ".join(m.group(1).split()) + "]", block, flags=re.S)
    for name in _declared():
        assert name in doc, f"{name} missing from the integration guide"
    kinds = {"P": ctypes.c_void_p, "I64": ctypes.c_int64, "I": ctypes.c_int, "F": ctypes.c_float}
    bound = re.findall(r"lib\.(tq_\w+)\.argtypes = \[([^\]]*)\]", block)
    assert len(bound) >= 20
    for name, args in bound:
        args = [a.strip() for a in args.split(",") if a.strip()]
        want = N.SIGNATURES[name]
        assert len(args) == len(want), (name, len(args), len(want))
        for i, (a, w) in enumerate(zip(args, want)):
            if a in kinds:
                assert kinds[a] is w, (name, i, a, w)


def test_decode_step_entries_check_arguments_on_the_host(lib):
    """The decode-step entry points reject bad calls before any CUDA call (fake,
    never-dereferenced pointers stand in for device memory)."""
    d, odd = ctypes.c_void_p(4096), ctypes.c_void_p(4096 + 8)
    # residual add + RMSNorm: dtype, width, null operands, strides, alignment; zero rows is a no-op
    assert lib.tq_add_rmsnorm(d, 64, None, 0, d, None, 0, d, 64, 2, 64, 1e-6, 7, None) == N.TQ_ERR_INVALID
    assert lib.tq_add_rmsnorm(d, 64, None, 0, d, None, 0, d, 64, 2, 60, 1e-6, 0, None) == N.TQ_ERR_INVALID
    assert b"multiple of 8" in lib.tq_last_error()
    assert lib.tq_add_rmsnorm(d, 64, None, 0, d, None, 0, d, 64, 0, 64, 1e-6, 0, None) == N.TQ_OK
    assert lib.tq_add_rmsnorm(None, 64, None, 0, d, None, 0, d, 64, 2, 64, 1e-6, 0, None) == N.TQ_ERR_INVALID
    assert lib.tq_add_rmsnorm(d, 64, d, 64, d, None, 0, d, 64, 2, 64, 1e-6, 0, None) == N.TQ_ERR_INVALID  # no resid_out
    assert lib.tq_add_rmsnorm(d, 32, None, 0, d, None, 0, d, 64, 2, 64, 1e-6, 0, None) == N.TQ_ERR_INVALID
    assert b"row stride" in lib.tq_last_error()
    assert lib.tq_add_rmsnorm(odd, 64, None, 0, d, None, 0, d, 64, 2, 64, 1e-6, 0, None) == N.TQ_ERR_INVALID
    assert b"16-byte" in lib.tq_last_error()
    # SiLU * up + quantizer: at most 128 rows, strides at least k
    assert lib.tq_silu_mul_quant(d, d, 64, 129, 64, d, 64, d, 64, d, 0, None) == N.TQ_ERR_INVALID
    assert lib.tq_silu_mul_quant(d, d, 32, 4, 64, d, 64, d, 64, d, 0, None) == N.TQ_ERR_INVALID
    # decode attention: head_dim, heads per KV head, cache length, alignment
    a = N.AttnArgs(q=4096, k=4096, v=4096, cos=4096, sin=4096, k_cache=4096, v_cache=4096, pos=4096, ws_m=4096,
                   ws_l=4096, ws_o=4096, err=0, ld_q=1024, ld_k=256, ld_v=256, B=4, Hq=8, Hkv=2, D=128, L=64, S=2,
                   scale_log2=0.1, reserved=0)
    assert lib.tq_attn_decode(None, d, 1024, None, 0, None, 0, None) == N.TQ_ERR_INVALID
    for field, value, code in (("D", 96, N.TQ_ERR_UNSUPPORTED), ("Hq", 32, N.TQ_ERR_UNSUPPORTED),
                               ("L", 0, N.TQ_ERR_INVALID), ("k_cache", 4104, N.TQ_ERR_INVALID),
                               ("ld_q", 1020, N.TQ_ERR_INVALID)):
        bad = N.AttnArgs.from_buffer_copy(a)
        setattr(bad, field, value)
        assert lib.tq_attn_decode(ctypes.byref(bad), d, 1024, None, 0, None, 0, None) == code, field
    assert lib.tq_attn_decode(ctypes.byref(a), d, 512, None, 0, None, 0, None) == N.TQ_ERR_INVALID  # ld_out < Hq*D
    # greedy pick: row count, vocabulary within the row stride
    assert lib.tq_greedy_pick(d, 128, 0, 128, 0, d, None, None, None, 0, 0, d, 0, None) == N.TQ_ERR_INVALID
    assert lib.tq_greedy_pick(d, 100, 2, 128, 0, d, None, None, None, 0, 0, d, 0, None) == N.TQ_ERR_INVALID
