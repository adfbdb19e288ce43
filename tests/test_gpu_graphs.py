"""The library inside CUDA graphs, as the engine uses it (inference/engine.py:337-360): every
call launches on the current stream and allocates only through PyTorch, so a captured step
replays on new inputs and equals the same calls run eagerly, bit for bit."""

import pytest
import torch

import jeeves_b200 as gdn
from jeeves_b200 import fla_inplace
from tests.helpers import gdn_inputs, same_bits

pytestmark = pytest.mark.gpu

H, HV = 4, 8
LENS = [70, 130, 1, 64]


def _inputs(seed):
    gen = torch.Generator().manual_seed(seed)
    T = sum(LENS)
    q, k, v, g, beta, _ = gdn_inputs(seed, 1, T, H, HV)
    dq, dk, dv, dg, db, _ = gdn_inputs(seed + 1, 6, 1, H, HV)
    vq, vk, vv, vg, vb, _ = gdn_inputs(seed + 2, 3, 4, H, HV)
    C = 2 * H * 128 + HV * 128
    x = dict(q=q, k=k, v=v, g=g, beta=beta, h0=torch.randn(len(LENS), HV, 128, 128, generator=gen) * 0.02,
             dq=dq, dk=dk, dv=dv, dg=dg, db=db, ds=torch.randn(6, HV, 128, 128, generator=gen) * 0.02,
             vq=vq, vk=vk, vv=vv, vg=vg, vb=vb, vs=torch.randn(3, HV, 128, 128, generator=gen) * 0.02,
             acc=torch.tensor([1, 4, 2]),
             vz=torch.randn(3, 4, HV, 128, generator=gen).to(torch.bfloat16),
             vqkv=(torch.randn(3, 4, C, generator=gen) * 2).to(torch.bfloat16),
             vcs=torch.randn(2, 3, C, 3, generator=gen).to(torch.bfloat16),
             qkv=(torch.randn(1, T, C, generator=gen) * 2).to(torch.bfloat16),
             w=(torch.randn(C, 4, generator=gen) * 0.5).to(torch.bfloat16),
             z=torch.randn(T * HV, 128, generator=gen).to(torch.bfloat16),
             nw=(torch.rand(128, generator=gen) + 0.5).to(torch.bfloat16),
             graw=(torch.randn(1, T, 2 * HV, generator=gen) * 3).to(torch.bfloat16),
             dt=torch.randn(HV, generator=gen), rate=-torch.rand(HV, generator=gen).exp(),
             valid=torch.rand(1, T, generator=gen) < 0.9,
             # the drafter side: mask-row attention over a key cache, rotary, rotate-into-cache
             aq=torch.randn(2, 12, HV, 128, generator=gen).to(torch.bfloat16),
             kc=torch.randn(3, 200, HV, 128, generator=gen).to(torch.bfloat16),
             vc=torch.randn(3, 200, HV, 128, generator=gen).to(torch.bfloat16),
             amask=torch.where(torch.rand(2, 1, 12, 192, generator=gen) < 0.7, 0.0, float("-inf")).to(torch.bfloat16),
             rx=torch.randn(2, 3, HV, 128, generator=gen).to(torch.bfloat16),
             rcos=torch.randn(2, 3, 32, generator=gen), rsin=torch.randn(2, 3, 32, generator=gen),
             ck=torch.randn(2, 2, HV, 128, generator=gen).to(torch.bfloat16),
             cm=torch.randn(2, 2, 3 * HV * 128, generator=gen).to(torch.bfloat16),
             kcache=torch.randn(3, 64, HV, 128, generator=gen).to(torch.bfloat16),
             vcache=torch.randn(3, 64, HV, 128, generator=gen).to(torch.bfloat16),
             rows=torch.tensor([[2, 2], [0, 0]]), positions=torch.tensor([[5, 6], [11, 12]]))
    return {name: t.cuda() for name, t in x.items()}


def _step(x, cu):
    y = gdn.causal_conv1d(x["qkv"], x["w"], cu_seqlens=cu)
    beta_g, g_g = gdn.delta_gates(x["graw"][..., :HV], x["graw"][..., HV:], x["dt"], x["rate"], x["valid"])
    o, ht = gdn.gated_delta_rule_chunk(x["q"], x["k"], x["v"], x["g"], x["beta"], initial_state=x["h0"],
                                       output_final_state=True, cu_seqlens=cu)
    out = gdn.gated_rms_norm(o.view(-1, 128), x["z"], x["nw"])
    od = fla_inplace.gated_delta_rule_step_inplace(x["dq"], x["dk"], x["dv"], x["dg"], x["db"], x["ds"])
    ov, snaps = gdn.gated_delta_rule_verify(x["vq"], x["vk"], x["vv"], x["vg"], x["vb"], x["vs"])
    # the tensor-core block verify, plain and with the gated norm fused, then its delta commit
    ob, db = gdn.gated_delta_rule_verify_deltas(x["vq"], x["vk"], x["vv"], x["vg"], x["vb"], x["vs"])
    yb, _ = gdn.gated_delta_rule_verify_deltas_gated_norm(x["vq"], x["vk"], x["vv"], x["vg"], x["vb"], x["vs"],
                                                          x["vz"], x["nw"])
    sc = x["vs"].clone()
    gdn.gated_delta_rule_delta_commit(x["vk"], x["vg"], db, sc, x["acc"])
    # the verify layer as one call (conv step, then the block verify as its programmatic dependent
    # with the gated norm) for two layers, then both layers' commits in one launch and the conv states'
    C = x["w"].shape[0]
    ext = torch.empty(2, 3, C, 3 + 4, dtype=torch.bfloat16, device="cuda")
    layer_states, pending, ys = [x["vs"].clone(), sc.clone()], [], []
    for l in range(2):
        yl, pl = gdn.verify_layer_step(x["vqkv"], x["vcs"][l], x["w"], x["vg"], x["vb"], layer_states[l], x["vz"],
                                       x["nw"], H, ext_out=ext[l], deltas=torch.empty(3, 4, HV, 128, device="cuda"))
        ys.append(yl)
        pending.append(pl)
    gdn.verify_layers_commit(pending, layer_states, x["acc"], ext=ext, conv_states=x["vcs"])
    gdn.gated_delta_rule_rollback(x["vs"], snaps, x["acc"])
    # the gates inside the prefill and the gated norm fused into the call
    og, hg = gdn.gated_delta_rule_chunk_gates(x["q"], x["k"], x["v"], x["graw"][..., :HV], x["graw"][..., HV:],
                                              x["dt"], x["rate"], x["valid"], initial_state=x["h0"],
                                              output_final_state=True, cu_seqlens=cu)
    on, hn = gdn.gated_delta_rule_chunk_gated_norm(x["q"], x["k"], x["v"], x["g"], x["beta"], x["z"], x["nw"],
                                                   initial_state=x["h0"], output_final_state=True, cu_seqlens=cu)
    oa = gdn.decode_attention(x["aq"], x["kc"], x["vc"], x["amask"], 128 ** -0.5)
    orot = gdn.rotary(x["rx"], x["rcos"], x["rsin"])
    D3 = HV * 128
    qm, km, vm = (x["cm"][..., i * D3:(i + 1) * D3].view(2, 2, HV, 128) for i in range(3))
    qr = gdn.rotate_into_cache(x["ck"], x["ck"], qm, km, vm, x["rcos"][:, :2], x["rsin"][:, :2], x["rcos"][:, 1:],
                               x["rsin"][:, 1:], x["kcache"], x["vcache"], x["rows"], x["positions"], 40)
    return (y, beta_g, g_g, o, ht, out, od, ov, ob, db, yb, sc, *ys, *layer_states, ext, og, hg, on, hn, oa, orot,
            qr)


def test_captured_layer_step_replays_equal_to_eager():
    cu = torch.tensor([0] + torch.tensor(LENS).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    static = _inputs(1)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm up outside the capture, as PyTorch asks
        for _ in range(2):
            _step({name: t.clone() for name, t in static.items()}, cu)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = _step(static, cu)
    for seed in (5, 9):
        fresh = _inputs(seed)
        for name in static:
            static[name].copy_(fresh[name])
        graph.replay()
        eager = _step(fresh, cu)  # mutates fresh["ds"] and fresh["vs"] as the replay mutated static's
        torch.cuda.synchronize()
        for a, b in zip(outs, eager):
            assert same_bits(a, b)
        assert same_bits(static["ds"], fresh["ds"]) and same_bits(static["vs"], fresh["vs"])
        assert same_bits(static["vcs"], fresh["vcs"])
        assert same_bits(static["kcache"], fresh["kcache"]) and same_bits(static["vcache"], fresh["vcache"])
    del graph
