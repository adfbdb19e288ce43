"""The reference's own code on the GPU with this library installed: ``GatedDeltaNet.forward``
(model/model.py:453-517) in prefill without a cache, with the growing ``Cache`` and with the
``StaticCache`` decode branch, and the engine's ``delta_extend`` / ``delta_outputs`` /
``delta_commit`` and ``conv_step`` (inference/engine.py:241-258, :427-430). Each runs the
reference's functions unchanged; ``install`` routes their fla calls to this library. The same
code on CPU tensors takes the reference's eager path and is the comparison, within the bounds the
tests of the kernels use (bf16 outputs max-abs 2e-2; fp32 states 1e-3 relative after a chunked
prefill, 1e-5 after recurrent steps).

The reference is imported from ``JEEVES_REFERENCE`` or the repository's ``baseline/_ref``
install; without either the tests print why and skip."""

import copy
import os
import sys
import types

import pytest
import torch

import jeeves_b200 as gdn
from tests.helpers import maxabs, rel, same_bits

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
O_TOL, S_TOL_CHUNK, S_TOL_STEP = 2e-2, 1e-3, 1e-5


def _reference_path():
    for cand in (os.environ.get("JEEVES_REFERENCE"), os.path.join(ROOT, "baseline", "_ref")):
        if cand and os.path.isfile(os.path.join(cand, "model", "model.py")):
            return cand
    return None


@pytest.fixture(scope="module")
def ref():
    path = _reference_path()
    if path is None:
        print("reference not installed (set JEEVES_REFERENCE or install it into baseline/_ref): skipping")
        pytest.skip("reference package not present")
    if path not in sys.path:
        sys.path.append(path)
    import model.model as mm
    from model.config import LINEAR, Qwen3_5_9BConfig, hybrid_layer_types

    engine = None
    try:
        import inference.engine as engine
    except Exception as e:  # the engine's own imports; the model tests still run
        print(f"inference.engine not importable: {type(e).__name__}: {e}")
    handle = gdn.install(mm, *(m for m in (engine,) if m is not None))
    cfg = Qwen3_5_9BConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
                           layer_types=hybrid_layer_types(4, 4), num_attention_heads=2, num_key_value_heads=1,
                           head_dim=64, linear_num_key_heads=2, linear_num_value_heads=4)
    assert cfg.layer_types[0] == LINEAR
    yield types.SimpleNamespace(mm=mm, engine=engine, cfg=cfg)
    handle.uninstall()


def _layer(ref, seed):
    torch.manual_seed(seed)
    layer = ref.mm.GatedDeltaNet(ref.cfg, 0)
    # a slower decay than the init's A in (0, 16), so that state carries over whole prompts
    with torch.no_grad():
        layer.A_log.uniform_(-4.0, 0.0)
    return layer.to(torch.bfloat16).eval()


def _hooked(layer):
    """The GDN output (the gated norm's input) of every forward call."""
    seen = []
    layer.norm.register_forward_hook(lambda mod, args, out: seen.append(args[0].detach().clone()))
    return seen


@torch.no_grad()
def test_gated_delta_net_prefill_without_cache(ref):
    cpu = _layer(ref, 0)
    gpu = copy.deepcopy(cpu).cuda()
    seen_c, seen_g = _hooked(cpu), _hooked(gpu)
    x = torch.randn(2, 150, ref.cfg.hidden_size, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    y_c = cpu(x)
    y_g = gpu(x.cuda())
    assert maxabs(seen_g[0], seen_c[0]) < O_TOL
    assert rel(y_g, y_c) < O_TOL


@torch.no_grad()
def test_gated_delta_net_growing_cache_prefill_then_steps(ref):
    """The reference's growing Cache: a prompt (chunked prefill with the final state), a second
    prompt part resumed from that state, then single-token steps (conv step + recurrent step)."""
    cpu = _layer(ref, 2)
    gpu = copy.deepcopy(cpu).cuda()
    seen_c, seen_g = _hooked(cpu), _hooked(gpu)
    cache_c, cache_g = ref.mm.Cache(ref.cfg.num_hidden_layers), ref.mm.Cache(ref.cfg.num_hidden_layers)
    gen = torch.Generator().manual_seed(3)
    parts = [torch.randn(2, T, ref.cfg.hidden_size, generator=gen).to(torch.bfloat16) for T in (70, 33, 1, 1, 1)]
    for i, x in enumerate(parts):
        cpu(x, cache_c)
        gpu(x.cuda(), cache_g)
        assert maxabs(seen_g[i], seen_c[i]) < O_TOL, i
        tol = S_TOL_CHUNK if i < 2 else S_TOL_CHUNK + S_TOL_STEP
        assert rel(cache_g.rec[0], cache_c.rec[0]) < tol, i
        # the conv state holds the pre-conv projection, a bf16 matmul on each side
        assert rel(cache_g.conv[0], cache_c.conv[0]) < 1e-2, i


@torch.no_grad()
def test_gated_delta_net_static_cache_decode_branch(ref):
    """StaticCache: the prefill branch (conv state copy, chunked prefill into rec), then the decode
    branch, whose fla_inplace step updates rec in place (model/model.py:496-499)."""
    cpu = _layer(ref, 4)
    gpu = copy.deepcopy(cpu).cuda()
    seen_c, seen_g = _hooked(cpu), _hooked(gpu)
    B, T = 3, 64
    sc_c = ref.mm.StaticCache(ref.cfg, B, 80, torch.device("cpu"), torch.bfloat16)
    sc_g = ref.mm.StaticCache(ref.cfg, B, 80, torch.device("cuda"), torch.bfloat16)
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(B, T, ref.cfg.hidden_size, generator=gen).to(torch.bfloat16)
    cpu(x, sc_c)
    gpu(x.cuda(), sc_g)
    for sc in (sc_c, sc_g):
        sc.finish_prefill(T, None)
    assert maxabs(seen_g[0], seen_c[0]) < O_TOL
    assert rel(sc_g.rec[0], sc_c.rec[0]) < S_TOL_CHUNK
    rec_ptr = sc_g.rec[0].data_ptr()
    for i in range(4):
        xt = torch.randn(B, 1, ref.cfg.hidden_size, generator=gen).to(torch.bfloat16)
        cpu(xt, sc_c)
        gpu(xt.cuda(), sc_g)
        assert maxabs(seen_g[1 + i], seen_c[1 + i]) < O_TOL, i
        assert rel(sc_g.conv[0], sc_c.conv[0]) < 1e-2, i
    assert sc_g.rec[0].data_ptr() == rec_ptr  # updated in place
    assert rel(sc_g.rec[0], sc_c.rec[0]) < S_TOL_CHUNK + S_TOL_STEP


@torch.no_grad()
def test_engine_delta_extend_outputs_commit(ref):
    """The engine's delta functions (called on a stand-in for the engine: they only read
    ``self.metal``), on CUDA tensors against the same calls on CPU tensors: a committed prefill, the
    outputs of 5 verified tokens without a state write, then the commit of 0-5 accepted tokens."""
    if ref.engine is None:
        pytest.skip("inference.engine is not importable here")
    E = ref.engine.Engine
    me = types.SimpleNamespace(metal=False)
    B, HV, D = 4, 4, 128
    gen = torch.Generator().manual_seed(6)

    def inputs(T):
        q, k = (torch.nn.functional.normalize(torch.randn(B, T, HV, D, generator=gen), dim=-1).to(torch.bfloat16)
                for _ in range(2))
        v = torch.randn(B, T, HV, D, generator=gen).to(torch.bfloat16)
        g = -torch.exp(torch.randn(B, T, HV, generator=gen) * 0.5 - 3.0)
        beta = torch.sigmoid(torch.randn(B, T, HV, generator=gen)).to(torch.bfloat16)
        return q, k, v, g, beta

    state_c = torch.randn(B, HV, D, D, generator=gen) * 0.02
    state_g = state_c.cuda()
    prompt = inputs(90)
    o_c = E.delta_extend(me, *prompt, state_c, True)
    o_g = E.delta_extend(me, *(t.cuda() for t in prompt), state_g, True)
    assert maxabs(o_g, o_c) < O_TOL
    assert rel(state_g, state_c) < S_TOL_CHUNK
    state_g.copy_(state_c)  # from here on both sides start from the same bits
    drafted = inputs(5)
    o_c = E.delta_outputs(me, *drafted, state_c)
    before = state_g.clone()
    o_g = E.delta_outputs(me, *(t.cuda() for t in drafted), state_g)
    assert maxabs(o_g, o_c) < O_TOL
    assert same_bits(state_g, before)
    accepted = torch.tensor([0, 1, 3, 5])
    q, k, v, g, beta = drafted
    E.delta_commit(me, k, v, g, beta, state_c, accepted)
    E.delta_commit(me, k.cuda(), v.cuda(), g.cuda(), beta.cuda(), state_g, accepted.cuda())
    assert rel(state_g, state_c) < S_TOL_STEP
    assert same_bits(state_g[0], before[0])


@torch.no_grad()
def test_engine_conv_step_and_gates(ref):
    """``conv_step`` as the engine imports it (ext written to a slice of its stacked buffer) and
    ``delta_gates``, on CUDA against CPU."""
    if ref.engine is None:
        pytest.skip("inference.engine is not importable here")
    cfg = ref.cfg
    B, T, C, taps = 3, 5, cfg.linear_conv_dim, cfg.linear_conv_kernel_dim
    gen = torch.Generator().manual_seed(7)
    state = torch.randn(B, C, taps, generator=gen).to(torch.bfloat16)
    qkv = torch.randn(B, T, C, generator=gen).to(torch.bfloat16)
    w = (torch.randn(C, 1, taps, generator=gen) * 0.5).to(torch.bfloat16)
    dims = (cfg.linear_key_dim, cfg.linear_value_dim, cfg.linear_key_head_dim, cfg.linear_value_head_dim)
    ext_c = torch.empty(B, C, taps + T, dtype=torch.bfloat16)
    ext_g = torch.empty(2, B, C, taps + T, dtype=torch.bfloat16, device="cuda")[1]
    got = ref.engine.conv_step(state.cuda(), qkv.cuda(), w.cuda(), *dims, ext_out=ext_g)
    want = ref.engine.conv_step(state, qkv, w, *dims, ext_out=ext_c)
    assert same_bits(ext_g, ext_c)
    for a, b in zip(got[1:], want[1:]):
        assert maxabs(a, b) <= 2 ** -6 * max(1.0, b.abs().max().item())  # SiLU may round one ulp apart
    b_in = torch.randn(B, T, cfg.linear_num_value_heads, generator=gen).to(torch.bfloat16)
    a_in = torch.randn(B, T, cfg.linear_num_value_heads, generator=gen).to(torch.bfloat16)
    dt_bias = torch.rand(cfg.linear_num_value_heads, generator=gen)
    rate = -torch.rand(cfg.linear_num_value_heads, generator=gen) * 8
    beta_g, g_g = ref.engine.delta_gates(b_in.cuda(), a_in.cuda(), dt_bias.cuda(), rate.cuda())
    beta_c, g_c = ref.engine.delta_gates(b_in, a_in, dt_bias, rate)
    assert maxabs(beta_g, beta_c) <= 2 ** -8  # CPU and CUDA sigmoid may round one bf16 ulp apart
    assert rel(g_g, g_c) < 1e-6
