"""GPU parity of the fused decode layer against the composition of the oracle's ops."""

import pytest
import torch

import jeeves_b200 as gdn
import oracle
from tests.helpers import maxabs, rel, same_bits

pytestmark = pytest.mark.gpu


def reference_layer(qkv, conv_state, w, g, beta, state, z, nw, H, HV):
    B, C = qkv.shape
    y = oracle.causal_conv1d_step(qkv, conv_state, w)  # updates conv_state
    kd = H * 128
    q = y[:, :kd].reshape(B, 1, H, 128)
    k = y[:, kd:2 * kd].reshape(B, 1, H, 128)
    v = y[:, 2 * kd:].reshape(B, 1, HV, 128)
    o, S = oracle.recurrent_gated_delta_rule(q, k, v, g.reshape(B, 1, HV), beta.reshape(B, 1, HV),
                                             initial_state=state, output_final_state=True)
    out = oracle.gated_rms_norm(o.reshape(-1, 128), z.reshape(-1, 128), nw).reshape(B, HV, 128)
    return out, S


@pytest.mark.parametrize("B,H,HV,taps", [(4, 16, 32, 4), (3, 2, 4, 3)])
def test_decode_layer_matches_composition(B, H, HV, taps):
    gen = torch.Generator().manual_seed(B * 10 + taps)
    C = 2 * H * 128 + HV * 128
    qkv = (torch.randn(B, C, generator=gen) * 2).to(torch.bfloat16)
    cs = torch.randn(B, C, taps, generator=gen).to(torch.bfloat16)
    w = (torch.randn(C, 4, generator=gen) * 0.5).to(torch.bfloat16)
    g = -torch.exp(torch.randn(B, HV, generator=gen) * 0.5 - 3.0)
    beta = torch.sigmoid(torch.randn(B, HV, generator=gen)).to(torch.bfloat16)
    state = torch.randn(B, HV, 128, 128, generator=gen) * 0.02
    z = torch.randn(B, HV, 128, generator=gen).to(torch.bfloat16)
    nw = (torch.rand(128, generator=gen) + 0.5).to(torch.bfloat16)
    cs_ref = cs.clone()
    if taps == 4:
        out_ref, S_ref = reference_layer(qkv, cs_ref, w, g, beta, state, z, nw, H, HV)
    else:  # the eager step keeps K taps; with 3 live taps the state holds the last 3 inputs
        full = torch.cat([torch.zeros(B, C, 1, dtype=cs.dtype), cs], dim=-1)
        out_ref, S_ref = reference_layer(qkv, full, w, g, beta, state, z, nw, H, HV)
        cs_ref = full[..., 1:]
    cs_gpu, st_gpu = cs.cuda(), state.cuda()
    out = gdn.decode_layer_step(qkv.cuda(), cs_gpu, w.cuda(), g.cuda(), beta.cuda(), st_gpu, z.cuda(), nw.cuda(), H)
    assert same_bits(cs_gpu, cs_ref)
    assert rel(st_gpu, S_ref) < 1e-5
    assert maxabs(out, out_ref) < 2e-2
    assert (out.cpu() != out_ref).float().mean().item() < 0.02
