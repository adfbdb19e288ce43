"""The reference's inference engine (inference/engine.py), unchanged, running its speculative decode
on this library: a tiny random-weight hybrid model of the Qwen3.5 shape (3 gated-delta layers with
2 key / 4 value heads of 128, 1 attention layer) and its drafter view go through ``Engine`` with
``install(model.model, inference.engine)``; the prompt prefill (``extend``) and the decode cycles
(``cycle``: conv step, delta gates, verify outputs, drafter mask-row attention, rotate-into-cache,
commit) run under the engine's own CUDA graphs. The check follows the reference's ``compare_ar``
(inference/bench.py:78-105): every chain must equal greedy autoregressive decoding of the same
model (``generate``), except from a step where greedy decoding itself is a tie in bf16 (the two
best logits within two units in the last place), after which the chains may part.

The engine loads weights through ``load_export`` and ``load_file``; the test hands it the random
model, the drafter's state and a stand-in for the tokenizer's ids instead (no checkpoint is
present). The reference comes from ``JEEVES_REFERENCE`` or ``baseline/_ref``; without it the test
prints why and skips."""

import math
import os
import sys
import types

import pytest
import torch

import jeeves_b200 as gdn
from jeeves_b200 import integration

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _reference_path():
    for cand in (os.environ.get("JEEVES_REFERENCE"), os.path.join(ROOT, "baseline", "_ref")):
        if cand and os.path.isfile(os.path.join(cand, "inference", "engine.py")):
            return cand
    return None


def _bf16_ulp(x: float) -> float:
    return 2.0 ** (math.floor(math.log2(abs(x))) - 7) if x else 2.0 ** -133


@torch.no_grad()
def test_engine_speculative_decode_matches_greedy_autoregressive(monkeypatch):
    path = _reference_path()
    if path is None:
        print("reference not installed (set JEEVES_REFERENCE or install it into baseline/_ref): skipping")
        pytest.skip("reference package not present")
    if path not in sys.path:
        sys.path.append(path)
    import inference.engine as eng
    import model.model as mm
    from drafter.view import DrafterView
    from model.config import LINEAR, Qwen3_5_9BConfig, hybrid_layer_types

    calls = {}
    for name in ("gated_delta_rule_chunk", "gated_delta_rule_step", "_conv_step", "_decode_attention", "_delta_gates"):
        fn = getattr(integration, name)

        def counted(*a, _fn=fn, _name=name, **k):
            calls[_name] = calls.get(_name, 0) + 1
            return _fn(*a, **k)

        monkeypatch.setattr(integration, name, counted)
    handle = gdn.install(mm, eng)
    try:
        # the attention layer keeps one key head per query head: torch 2.11's memory-efficient SDPA
        # (the engine's backend) takes no grouped heads
        cfg = Qwen3_5_9BConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
                               layer_types=hybrid_layer_types(4, 4), num_attention_heads=2, num_key_value_heads=2,
                               head_dim=128, linear_num_key_heads=2, linear_num_value_heads=4, eos_token_id=7)
        torch.manual_seed(0)
        base = mm.Qwen3_5ForCausalLM(cfg)
        for p in base.parameters():
            if p.dim() >= 2:
                p.normal_(0, 0.05)
        for layer in base.model.layers:
            if layer.layer_type == LINEAR:
                layer.linear_attn.A_log.uniform_(-3, 0)  # decays that carry state over the prompt
        base.model.embed_tokens.weight.normal_(0, 1.0)
        base.lm_head.weight.normal_(0, 0.3)
        base = base.to(torch.bfloat16).cuda()
        drafter_state = {k: v for k, v in DrafterView(base, block=4).state_dict().items() if not k.startswith("base.")}
        encoder = types.SimpleNamespace(think_end_id=7, pad_id=0, opt_end_id=1, empty_think=[2, 3], banned_ids=[4])
        monkeypatch.setattr(eng, "load_export", lambda p, device=None: (base, None, encoder))
        monkeypatch.setattr(eng, "load_file", lambda p, device=None: {k: v.to(device) for k, v in drafter_state.items()})
        E = eng.Engine("model", "drafter", block=4, precision="bf16", max_rows=4, max_len=512, device="cuda")

        gen = torch.Generator().manual_seed(1)
        prompts = [torch.randint(10, 500, (n,), generator=gen).tolist() for n in (17, 40, 29)]
        B, cap = len(prompts), 40
        # the engine's flow for token prompts (Engine.group without the tokenizer's text steps)
        E.reset(E.decode_rows(B))
        h = E.extend(prompts, [0] * B, commit=True)
        last = h[torch.arange(B, device="cuda"), torch.tensor([len(p) - 1 for p in prompts], device="cuda")]
        first = (E.vocab_logits(last) + E.bias).argmax(-1)
        chains, _ = E.decode(B, prompts, first, [cap] * B)
        assert len(E.cycle_graphs) >= 1 and len(E.extend_graphs) >= 1  # the engine ran its CUDA graphs

        for b, p in enumerate(prompts):
            ref = base.generate(torch.tensor(p, device="cuda")[None], max_new_tokens=cap, temperature=0.0,
                                eos_token_id=E.eos, logit_bias=E.bias.float())[0, len(p):].tolist()
            if E.eos in ref:
                ref = ref[:ref.index(E.eos) + 1]
            m = 0
            while m < min(len(ref), len(chains[b])) and chains[b][m] == ref[m]:
                m += 1
            if m == len(ref) == len(chains[b]):
                continue
            assert m < min(len(ref), len(chains[b])), (b, m, len(ref), len(chains[b]))
            # greedy's choice at the first difference is a bf16 tie with the engine's
            lg = base(torch.tensor(p + ref[:m], device="cuda")[None]).logits[0, -1].float() + E.bias.float()
            best = float(lg.max())
            assert best - float(lg[chains[b][m]]) <= 2 * _bf16_ulp(best), (b, m, best, float(lg[chains[b][m]]))
        for name in ("gated_delta_rule_chunk", "gated_delta_rule_step", "_conv_step", "_decode_attention",
                     "_delta_gates"):
            assert calls.get(name, 0) > 0, (name, calls)
    finally:
        handle.uninstall()
