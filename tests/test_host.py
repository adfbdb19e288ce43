"""CPU checks of the Python host layer: signatures, validation and the reference hook-up."""

import os
import sys
import types

import pytest
import torch

import jeeves_b200 as gdn
from jeeves_b200 import integration

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# the reference checkout or install: JEEVES_REFERENCE, else the repository's baseline/_ref
REFERENCE = os.environ.get("JEEVES_REFERENCE") or os.path.join(ROOT, "baseline", "_ref")


def test_cpu_tensors_are_rejected_not_computed():
    q = torch.zeros(1, 2, 1, 128, dtype=torch.bfloat16)
    g = torch.zeros(1, 2, 1)
    with pytest.raises(ValueError, match="CUDA"):
        gdn.gated_delta_rule_chunk(q, q, q, g, g.to(torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):
        gdn.gated_delta_rule_step(q, q, q, g, g.to(torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):
        gdn.causal_conv1d(torch.zeros(1, 4, 8, dtype=torch.bfloat16), torch.zeros(8, 4, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):
        gdn.gated_rms_norm(torch.zeros(2, 128, dtype=torch.bfloat16), torch.zeros(2, 128, dtype=torch.bfloat16),
                           torch.ones(128, dtype=torch.bfloat16))


def fake_reference_module():
    m = types.ModuleType("fake_model")
    m._AVAILABLE = {"gdn": False, "causal_conv1d": False, "rms_norm_gated": False, "triton_inference": False}
    m._ENABLED_BY_ENV = True
    m.KERNELS = dict(m._AVAILABLE)
    m._on = lambda name, x: m.KERNELS[name] and x.is_cuda
    m.calls = []
    m.eager_conv_step = lambda *a, **k: m.calls.append("eager_conv") or "eager"
    m.conv_step = lambda *a, **k: m.calls.append("conv") or "conv"
    m.gated_delta_rule_advance_inplace = lambda *a, **k: m.calls.append("advance") or None
    m.gated_delta_rule_chunk = lambda *a, **k: "chunk"
    m.gated_delta_rule_step = lambda *a, **k: "step"
    m.causal_conv1d = lambda *a, **k: "c1d"
    m.causal_conv1d_step = lambda *a, **k: "c1ds"
    m.delta_gates = lambda *a, **k: m.calls.append("gates") or "gates"
    m.fla_inplace = None
    return m


def test_install_sets_hooks_and_restores():
    m = fake_reference_module()
    engine = types.ModuleType("fake_engine")
    engine.conv_step = m.conv_step
    engine.gated_delta_rule_advance_inplace = m.gated_delta_rule_advance_inplace
    engine.delta_gates = m.delta_gates
    before = (m._AVAILABLE, m.KERNELS, m.conv_step, engine.conv_step, m.delta_gates, engine.delta_gates)
    h = gdn.install(m, engine)
    assert m._fla_chunk_gdr is integration.fla_chunk_gated_delta_rule
    assert m._fla_recurrent_gdr is integration.fla_fused_recurrent_gated_delta_rule
    assert m.fla_inplace is gdn.fla_inplace
    assert all(m.KERNELS[f] for f in integration.KERNEL_FAMILIES)
    assert engine.conv_step is m.conv_step and engine.delta_gates is m.delta_gates
    # CPU tensors keep the reference's own eager path
    cpu = torch.zeros(1, 1, 8, dtype=torch.bfloat16)
    assert m.conv_step(None, cpu, None, 2, 4, 1, 1) == "conv"
    m.gated_delta_rule_advance_inplace(cpu, cpu, None, None, None, None)
    assert m.delta_gates(cpu, cpu, None, None) == "gates"
    assert m.calls == ["conv", "advance", "gates"]
    h.uninstall()
    assert (m._AVAILABLE, m.KERNELS, m.conv_step, engine.conv_step, m.delta_gates, engine.delta_gates) == before
    assert not hasattr(m, "_fla_chunk_gdr")


def test_fla_adapters_require_in_kernel_l2norm():
    with pytest.raises(ValueError, match="use_qk_l2norm_in_kernel"):
        integration.fla_chunk_gated_delta_rule(None, None, None, use_qk_l2norm_in_kernel=False)


@pytest.mark.skipif(not os.path.isdir(os.path.join(REFERENCE, "model")), reason="reference checkout not present")
def test_install_into_reference_module():
    if REFERENCE not in sys.path:
        sys.path.append(REFERENCE)
    import model.model as ref
    h = gdn.install(ref)
    try:
        assert ref._fla_chunk_gdr is integration.fla_chunk_gated_delta_rule
        # on CPU the reference still runs its eager oracle through its own dispatcher
        x = torch.randn(1, 3, 2, 128)
        g = -torch.rand(1, 3, 2)
        b = torch.rand(1, 3, 2)
        o, S = ref.gated_delta_rule_chunk(x, x, x, g, b, output_final_state=True)
        assert o.shape == (1, 3, 2, 128) and S.shape == (1, 2, 128, 128)
        raw = torch.randn(2, 3, 4).to(torch.bfloat16)
        beta, gg = ref.delta_gates(raw, raw, torch.zeros(4), -torch.ones(4))
        assert beta.dtype == torch.bfloat16 and gg.dtype == torch.float32
    finally:
        h.uninstall()
