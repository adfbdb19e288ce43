"""The decode layer's no-allocation entry point, checked against the ordinary one.

gdn_decode_layer_noalloc exists for callers that cannot allocate device memory or pass the
library a buffer of their own: a plugin host or server that has handed every byte of device
memory to its own pool, a foreign-language binding with no device buffer to give, or code
that must not grow the process's device footprint after start-up. It keeps its scratch in a
fixed 4 MiB device array inside the library instead of taking a workspace argument.

Both entry points run the same kernels, so results must agree bit for bit. Two calls in a
row check that the shared array carries nothing over from one call into the next. This
file is named so that pytest collects it last.
"""

import ctypes

import pytest
import torch

from jeeves_b200 import _lib

H, HV, D, TAPS, K = 16, 32, 128, 3, 4
C = 2 * H * D + HV * D
SCRATCH_ELEMS = 1 << 21


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _inputs(B, seed):
    gen = torch.Generator().manual_seed(seed)
    dev = "cuda"
    return dict(
        qkv=(torch.randn(B, C, generator=gen) * 2).to(torch.bfloat16).to(dev),
        conv_state=torch.randn(B, C, TAPS, generator=gen).to(torch.bfloat16).to(dev),
        conv_w=(torch.randn(C, K, generator=gen) * 0.5).to(torch.bfloat16).to(dev),
        g=(-torch.exp(torch.randn(B, HV, generator=gen) * 0.5 - 3.0)).to(dev),
        beta=torch.sigmoid(torch.randn(B, HV, generator=gen)).to(torch.bfloat16).to(dev),
        state=(torch.randn(B, HV, D, D, generator=gen) * 0.02).to(dev),
        z=torch.randn(B, HV, D, generator=gen).to(torch.bfloat16).to(dev),
        norm_w=(torch.rand(D, generator=gen) + 0.5).to(torch.bfloat16).to(dev),
    )


def _call(lib, x, out, workspace=None):
    B = x["qkv"].shape[0]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    common = [_ptr(x["qkv"]), C, _ptr(x["conv_state"]), _ptr(x["conv_w"]), _ptr(x["g"]), _ptr(x["beta"]),
              _ptr(x["state"]), _ptr(x["z"]), _ptr(x["norm_w"]), _ptr(out)]
    tail = [B, H, HV, D, D, TAPS, K, D ** -0.5, 1e-6, stream]
    if workspace is None:
        return lib.gdn_decode_layer_noalloc(*common, *tail)
    return lib.gdn_decode_layer(*common, _ptr(workspace), *tail)


@pytest.mark.gpu
@pytest.mark.parametrize("B", [64, 256])
def test_noalloc_matches_workspace_entry_point_twice(B):
    lib = _lib.load()
    ref = _inputs(B, seed=B)
    mine = {k: v.clone() for k, v in ref.items()}
    workspace = torch.empty(B, C, dtype=torch.bfloat16, device="cuda")
    for step in range(2):  # the second call starts from the states the first one left
        out_ref = torch.empty(B, HV, D, dtype=torch.bfloat16, device="cuda")
        out_mine = torch.full((B, HV, D), float("nan"), dtype=torch.bfloat16, device="cuda")
        assert _call(lib, ref, out_ref, workspace) == _lib.OK
        assert _call(lib, mine, out_mine) == _lib.OK
        torch.cuda.synchronize()
        # same kernels on the same inputs: equal to the bit (tolerance 0)
        assert torch.equal(out_mine, out_ref), step
        assert torch.equal(mine["state"], ref["state"]), step
        assert torch.equal(mine["conv_state"], ref["conv_state"]), step
        # fresh token for the next call
        new_qkv = (torch.randn(B, C, generator=torch.Generator().manual_seed(100 + step)) * 2).to(torch.bfloat16)
        ref["qkv"].copy_(new_qkv)
        mine["qkv"].copy_(new_qkv)


def test_noalloc_rejects_requests_beyond_its_scratch():
    """batch * C above 2^21 bf16 values is refused before anything reaches the GPU."""
    lib = _lib.load()
    too_many = SCRATCH_ELEMS // C + 1
    status = lib.gdn_decode_layer_noalloc(16, C, 16, 16, 16, 16, 16, 16, 16, 16, too_many, H, HV, D, D, TAPS, K,
                                          D ** -0.5, 1e-6, None)
    assert status == _lib.ERR_SCRATCH
    assert "scratch" in _lib.status_text(status)
    with pytest.raises(ValueError, match="scratch"):
        _lib.check(status, "gdn_decode_layer_noalloc")
