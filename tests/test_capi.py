"""CPU checks of the C ABI: the library loads, exports every declared entry point, and
rejects bad arguments before touching a GPU."""

import ctypes
import os
import re

import pytest

from jeeves_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gdn_b200.h")


def declared():
    text = open(HEADER).read()
    return re.findall(r"GDN_API\s+[\w\s\*]+?\b(gdn_\w+)\s*\(", text)


def test_header_declares_entry_points():
    names = declared()
    assert "gdn_recurrent" in names and "gdn_conv_step" in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_binding_covers_exactly_the_header():
    assert set(_lib.SIGNATURES) == set(declared())


def test_status_strings_and_version():
    assert _lib.status_text(0) == "ok"
    assert "aligned" in _lib.status_text(_lib.ERR_ALIGN)
    assert _lib.load().gdn_abi_version() >= 1


def _recurrent(lib, **over):
    args = dict(q=None, k=16, v=16, qkv_dtype=_lib.BF16, g=16, beta=16, beta_dtype=_lib.BF16, state_in=None,
                state_out=None, snapshots=None, o=None, steps=None, cu=None, B=1, T=1, H=1, HV=1, Dk=128, Dv=128,
                strides=(128, 128, 128) * 3, scale=0.0884, stream=None)
    args.update(over)
    return lib.gdn_recurrent(args["q"], args["k"], args["v"], args["qkv_dtype"], args["g"], args["beta"],
                             args["beta_dtype"], args["state_in"], args["state_out"], args["snapshots"], args["o"],
                             args["steps"], args["cu"], args["B"], args["T"], args["H"], args["HV"], args["Dk"],
                             args["Dv"], *args["strides"], args["scale"], args["stream"])


def test_argument_checks_run_before_any_launch():
    lib = _lib.load()
    assert _recurrent(lib, qkv_dtype=7) == _lib.ERR_DTYPE
    assert _recurrent(lib, HV=3, H=2) == _lib.ERR_SHAPE
    assert _recurrent(lib, Dk=64) == _lib.ERR_UNSUPPORTED
    assert _recurrent(lib, k=None) == _lib.ERR_NULL
    assert _recurrent(lib, k=18) == _lib.ERR_ALIGN
    assert _recurrent(lib, strides=(128,) * 3 + (128, 129, 128) + (128,) * 3) == _lib.ERR_ALIGN
    assert _recurrent(lib, o=16, q=None) == _lib.ERR_NULL
    assert _recurrent(lib, steps=16, o=16, q=16) == _lib.ERR_SHAPE
    assert _recurrent(lib, B=0) == _lib.OK  # empty batch: nothing to launch
    assert lib.gdn_gated_rmsnorm(16, 16, 16, 16, 4, 64, 1e-6, None) == _lib.ERR_UNSUPPORTED
    assert lib.gdn_conv1d_silu(16, 0, 0, 16, 16, None, 1, 4, 12, 4, None) == _lib.ERR_SHAPE
    assert lib.gdn_conv_step(16, 16, 0, 0, 16, 16, 16, 16, 16, 1, 1, 4, 4, 33, 64, 16, 16, None) == _lib.ERR_SHAPE
    assert lib.gdn_snapshot_commit(16, 16, None, 2, 5, 4, 128, 128, None) == _lib.ERR_NULL


def _verify_layer(lib, **over):
    a = dict(qkv=16, sb=8192 * 5, st=8192, cs=16, cw=16, ext=16, q=16, k=16, v=16, g=16, beta=16, bd=_lib.BF16,
             state=16, z=16, nw=16, y=16, deltas=16, B=2, T=5, H=16, HV=32, Dk=128, Dv=128, taps=3, K=4)
    a.update(over)
    return lib.gdn_verify_layer_deltas(a["qkv"], a["sb"], a["st"], a["cs"], a["cw"], a["ext"], a["q"], a["k"], a["v"],
                                       a["g"], a["beta"], a["bd"], a["state"], a["z"], a["nw"], a["y"], a["deltas"],
                                       a["B"], a["T"], a["H"], a["HV"], a["Dk"], a["Dv"], a["taps"], a["K"], 0.0884,
                                       1e-6, None)


def test_verify_layer_call_checks_its_arguments_before_any_launch():
    lib = _lib.load()
    assert _verify_layer(lib, bd=9) == _lib.ERR_DTYPE
    assert _verify_layer(lib, HV=24, H=16) == _lib.ERR_SHAPE
    assert _verify_layer(lib, taps=3, K=5) == _lib.ERR_SHAPE
    assert _verify_layer(lib, Dv=64) == _lib.ERR_UNSUPPORTED
    assert _verify_layer(lib, T=9) == _lib.ERR_UNSUPPORTED  # the tensor-core block takes up to 8 tokens
    assert _verify_layer(lib, state=None) == _lib.ERR_NULL
    assert _verify_layer(lib, deltas=24) == _lib.ERR_ALIGN
    assert _verify_layer(lib, B=0) == _lib.OK and _verify_layer(lib, T=0) == _lib.OK  # nothing to launch


def test_layer_commit_checks_its_arguments_before_any_launch():
    lib = _lib.load()
    arr = ctypes.c_void_p * 2
    state_bytes = 2 * 32 * 128 * 128 * 4

    def commit(states, layers=2, B=2, **over):
        a = dict(kd=_lib.BF16, H=16, HV=32, Dk=128)
        a.update(over)
        return lib.gdn_delta_commit_layers(arr(*states), arr(16, 16), a["kd"], arr(16, 16), arr(16, 16), layers, 16, B,
                                           5, a["H"], a["HV"], a["Dk"], 128, 5 * 16 * 128, 16 * 128, 128, None)
    assert commit([16, 16 + state_bytes], kd=9) == _lib.ERR_DTYPE
    assert commit([16, 16 + state_bytes], Dk=64) == _lib.ERR_UNSUPPORTED
    assert commit([16, None]) == _lib.ERR_NULL
    assert commit([16, 16 + state_bytes - 16]) == _lib.ERR_SHAPE  # the two layers' states overlap
    assert commit([16, 24 + state_bytes]) == _lib.ERR_ALIGN
    assert commit([16, 16], layers=0) == _lib.OK and commit([16, 16], B=0) == _lib.OK


def test_status_mapping_to_exceptions():
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_SHAPE, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ERR_LAUNCH, "x")
    _lib.check(_lib.OK, "x")


def test_chunk_workspace_size_and_checks():
    """The prefill's workspace: its size rule, and a missing / short / misaligned one is refused."""
    lib = _lib.load()
    rec = 33792  # record bytes per (value head, chunk slot), then a 4-byte ready flag each

    def size(records, seqs=0):  # records, their flags, and the sequence order of a packed batch
        return records * rec + (records * 4 + 255) // 256 * 256 + (seqs * 4 + 255) // 256 * 256

    assert lib.gdn_chunk_prefill_workspace_size(1, 4096, 32, 0) == size(64 * 32)
    assert lib.gdn_chunk_prefill_workspace_size(3, 100, 4, 0) == size(3 * 2 * 4)
    assert lib.gdn_chunk_prefill_workspace_size(5, 300, 4, 1) == size((5 + 5) * 4, 5)  # ceil(T/64) + N slots
    args = [16, 16, 16, 16, 16, _lib.BF16, None, None, 16, None, 1, 64, 1, 1, 128, 128] + [128] * 9 + [0.088]
    need = lib.gdn_chunk_prefill_workspace_size(1, 64, 1, 0)
    assert lib.gdn_chunk_prefill(*args, None, need, None) == _lib.ERR_WORKSPACE
    assert lib.gdn_chunk_prefill(*args, 16, need - 16, None) == _lib.ERR_WORKSPACE
    assert lib.gdn_chunk_prefill(*args, 24, need, None) == _lib.ERR_ALIGN
    with pytest.raises(ValueError, match="workspace"):
        _lib.check(_lib.ERR_WORKSPACE, "gdn_chunk_prefill")
    # the norm-fused form checks its own pointers first, then the same workspace
    norm = lambda z, w, out, ws, n: lib.gdn_chunk_prefill_gated_norm(*args, z, w, 1e-6, out, ws, n, None)  # noqa: E731
    assert norm(None, 16, 16, 16, need) == _lib.ERR_NULL
    assert norm(16, 16, None, 16, need) == _lib.ERR_NULL
    assert norm(16, 8, 16, 16, need) == _lib.ERR_ALIGN
    assert norm(16, 16, 40, 16, need) == _lib.ERR_ALIGN
    assert norm(16, 16, 16, None, need) == _lib.ERR_WORKSPACE


def test_gate_entry_points_check_their_inputs():
    """The *_gates entry points refuse a missing gate struct, missing projections and a bad
    dt_bias dtype before any launch."""
    lib = _lib.load()
    qkv = [16, 16, 16]
    strides = [128] * 9
    good = _lib.GateInputs(16, 32, 16, 32, 16, _lib.F32, 16, None)
    no_a = _lib.GateInputs(16, 32, None, 32, 16, _lib.F32, 16, None)
    bad_dt = _lib.GateInputs(16, 32, 16, 32, 16, 7, 16, None)
    rec = lambda gates: lib.gdn_recurrent_gates(*qkv, _lib.BF16, gates, None, None, None, 16, None, None,  # noqa: E731
                                                1, 1, 1, 1, 128, 128, *strides, 0.088, None)
    assert rec(None) == _lib.ERR_NULL
    assert rec(ctypes.byref(no_a)) == _lib.ERR_NULL
    assert rec(ctypes.byref(bad_dt)) == _lib.ERR_DTYPE
    need = lib.gdn_chunk_prefill_workspace_size(1, 64, 1, 0)
    chunk = lambda gates, ws: lib.gdn_chunk_prefill_gates(*qkv, gates, None, None, 16, None, 1, 64, 1, 1,  # noqa: E731
                                                          128, 128, *strides, 0.088, ws, need, None)
    assert chunk(None, 16) == _lib.ERR_NULL
    assert chunk(ctypes.byref(no_a), 16) == _lib.ERR_NULL
    assert chunk(ctypes.byref(bad_dt), 16) == _lib.ERR_DTYPE
    assert chunk(ctypes.byref(good), None) == _lib.ERR_WORKSPACE


def test_attention_entry_points_check_their_inputs():
    lib = _lib.load()
    s3 = [128 * 4, 128 * 4, 128]
    args = lambda **kw: [kw.get("q", 16), *s3, 16, *s3, 16, *s3, kw.get("mask", 16), 64, 64, 16,  # noqa: E731
                         kw.get("B", 1), kw.get("R", 4), kw.get("H", 4), kw.get("Hkv", 4), kw.get("D", 128),
                         kw.get("L", 64), 1, 64, 0.1, None, 0, None]
    assert lib.gdn_decode_attention(*args(D=64)) == _lib.ERR_UNSUPPORTED
    assert lib.gdn_decode_attention(*args(R=65)) == _lib.ERR_UNSUPPORTED
    assert lib.gdn_decode_attention(*args(H=6)) == _lib.ERR_SHAPE
    assert lib.gdn_decode_attention(*args(L=65)) == _lib.ERR_SHAPE  # more keys than the cache holds
    assert lib.gdn_decode_attention(*args(mask=None)) == _lib.ERR_NULL
    assert lib.gdn_decode_attention(*args(q=24)) == _lib.ERR_ALIGN
    assert lib.gdn_decode_attention_workspace_size(2, 4, 64, 128) == 0  # one 64-key block: one range
    assert lib.gdn_decode_attention_workspace_size(64, 32, 4096, 128) == 0  # 2,048 (row, head) pairs: one range each
    assert lib.gdn_rotary(16, 16, 16, 16, 1, 1, 1, 128, 65, None) == _lib.ERR_SHAPE
    assert lib.gdn_rotary(None, 16, 16, 16, 1, 1, 1, 128, 32, None) == _lib.ERR_NULL
    assert lib.gdn_rotate_into_cache(16, 16, 16, 16, 16, 0, 0, 16, 16, 16, 16, None, 16, 0, 0, 16, 16, 0, 0, 16, 0,
                                     1, 1, 1, 1, 128, 32, None) == _lib.ERR_NULL


def test_probe_limit_is_checked():
    lib = _lib.load()
    assert lib.gdn_probe_bounded_wait(10, None) == _lib.ERR_SHAPE
    assert lib.gdn_probe_bounded_wait(10 ** 12, None) == _lib.ERR_SHAPE


def test_in_proj_conv_checks_its_inputs():
    lib = _lib.load()
    args = lambda **kw: [16, kw.get("ldx", 64), 16, 64, 16, None, 16, 24, None, kw.get("T", 10), kw.get("K", 64),  # noqa: E731
                         kw.get("N", 24), kw.get("C", 16), 1, kw.get("taps", 4), None]
    assert lib.gdn_in_proj_conv(*args(K=96)) == _lib.ERR_SHAPE        # hidden not a multiple of 64
    assert lib.gdn_in_proj_conv(*args(C=12)) == _lib.ERR_SHAPE        # channels not multiples of 8
    assert lib.gdn_in_proj_conv(*args(C=32)) == _lib.ERR_SHAPE        # more conv channels than outputs
    assert lib.gdn_in_proj_conv(*args(taps=3)) == _lib.ERR_UNSUPPORTED
    assert lib.gdn_in_proj_conv(*args(ldx=60)) == _lib.ERR_ALIGN
    assert lib.gdn_in_proj_conv(*args(T=0)) == _lib.OK


def test_fp8_workspace_sizes_and_checks():
    """The fp8 projection's workspaces: the base size holds the fp16 rows and their scales; the
    prefill size is never smaller (on a machine without a GPU no shape is planned onto CTA pairs,
    so the two agree); a workspace below the base size is rejected before any launch."""
    lib = _lib.load()
    T, K, N = 300, 256, 512
    base = lib.gdn_in_proj_fp8_workspace_size(T, K)
    assert base == (T * K * 2 + 255) // 256 * 256 + T * 4
    big = lib.gdn_in_proj_fp8_prefill_workspace_size(T, K, N, 0)
    assert big >= base
    assert big in (base, (base + 255) // 256 * 256 + N * K * 2)
    assert lib.gdn_in_proj_fp8_prefill_workspace_size(0, K, N, 0) == 0
    assert lib.gdn_in_proj_fp8_prefill_workspace_size(T, K, N, -1) == 0

    def call(ws_bytes, codes_stride=K):
        return lib.gdn_in_proj_conv_fp8(16, K, 16, codes_stride, 16, None, None, 16, N, None, 16, ws_bytes,
                                        T, K, N, 0, 1, 4, None)
    assert call(base - 1) == _lib.ERR_WORKSPACE
    assert call(base, codes_stride=K + 8) == _lib.ERR_ALIGN  # code rows must be 16-byte multiples
