"""GPU parity of the drafter's attention-side kernels: rotary and rotate-into-cache bit for bit
against the eager path (the comparison of model/triton_kernels_test.py:31-52 and :135-162), and
decode attention against the fp32 reference within the bounds the reference holds its own kernel
to (model/triton_kernels_test.py:104-132: mean error at most 1.25x, max error at most 2x that of
SDPA's kernel on the same bf16 inputs)."""

import pytest
import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

import jeeves_b200 as gdn
import oracle
from tests.helpers import same_bits

pytestmark = pytest.mark.gpu


def test_rotary_golden(golden):
    c = golden("rotary")
    y = gdn.rotary(c["x"].cuda(), c["cos"].cuda(), c["sin"].cuda())
    assert same_bits(y, c["y"])


@pytest.mark.parametrize("B,T,H,D", [(1, 4, 32, 128), (1, 12, 32, 128), (4, 16, 16, 256), (2, 190, 4, 256),
                                     (1, 1, 32, 128)])
def test_rotary_equals_eager(B, T, H, D):
    gen = torch.Generator().manual_seed(B * 1000 + T)
    x = torch.randn(B, T, H, D, generator=gen).to(torch.bfloat16)
    pos = (torch.arange(T)[None] + torch.randint(0, 8000, (B, 1), generator=gen)).float()[..., None]
    freqs = pos * torch.logspace(0, -7, 32)
    cos, sin = freqs.cos(), freqs.sin()
    assert same_bits(gdn.rotary(x.cuda(), cos.cuda(), sin.cuda()), oracle.apply_rotary(x, cos, sin))
    # cos for one row, broadcast over the batch
    assert same_bits(gdn.rotary(x.cuda(), cos[:1].cuda(), sin[:1].cuda()), oracle.apply_rotary(x, cos[:1], sin[:1]))


def test_rotate_into_cache_golden(golden):
    c = golden("rotate_into_cache")
    K, H, D = c["K"], c["k"].shape[2], c["k"].shape[3]
    merged = c["merged"].cuda()
    B, M = merged.shape[:2]
    qm, km, vm = (merged[..., i * H * D:(i + 1) * H * D].view(B, M, H, D) for i in range(3))
    kc, vc = c["k_cache"].cuda(), c["v_cache"].cuda()
    cos, sin = c["cos"].cuda(), c["sin"].cuda()
    q = gdn.rotate_into_cache(c["k"].cuda(), c["v"].cuda(), qm, km, vm, cos[:, :K], sin[:, :K], cos[:, K:], sin[:, K:],
                              kc, vc, c["rows"].cuda(), c["positions"].cuda(), c["tail"])
    assert same_bits(q, c["q_out"]) and same_bits(kc, c["k_cache_after"]) and same_bits(vc, c["v_cache_after"])


@pytest.mark.parametrize("B,K", [(1, 4), (4, 4), (2, 8)])
@pytest.mark.parametrize("shuffled", [False, True])
def test_rotate_into_cache_equals_eager(B, K, shuffled):
    gen = torch.Generator().manual_seed(B * 10 + K)
    H, D, nf, slots, tail = 32, 128, 32, 700, 512
    M = K * (K - 1)
    k, v = (torch.randn(B, K, H, D, generator=gen).to(torch.bfloat16) for _ in range(2))
    merged = torch.randn(B, M, 3 * H * D + 8, generator=gen).to(torch.bfloat16)
    positions = torch.randint(0, tail - K, (B, 1), generator=gen) + torch.arange(K)[None]
    freqs = torch.rand(B, K + M, 1, generator=gen) * 4000 * torch.logspace(0, -7, nf)
    cos, sin = freqs.cos(), freqs.sin()
    caches = [torch.randn(8, slots, H, D, generator=gen).to(torch.bfloat16) for _ in range(2)]
    rows = (torch.randperm(8, generator=gen)[:B] if shuffled else torch.arange(B))[:, None].expand(B, K)
    cos_rows = 1 if shuffled else B

    def run(mod, dev):
        mm = merged.to(dev)
        qm, km, vm = (mm[..., i * H * D:(i + 1) * H * D].view(B, M, H, D) for i in range(3))
        kc, vc = (t.clone().to(dev) for t in caches)
        c, s = cos[:cos_rows].to(dev), sin[:cos_rows].to(dev)
        q = mod.rotate_into_cache(k.to(dev), v.to(dev), qm, km, vm, c[:, :K], s[:, :K], c[:, K:], s[:, K:], kc, vc,
                                  rows.to(dev), positions.to(dev), tail)
        return q, kc, vc

    for got, want in zip(run(gdn, "cuda"), run(oracle, "cpu")):
        assert same_bits(got, want)


def _attention_case(seed, B, first_row, H, Hkv, D, Lw, K=4):
    """The engine's decode masks (as model/triton_kernels_test.py:104-121 builds them): row t < K
    sees the cache up to n + t; a mask row of block j sees the cache up to n + j and its block's
    tail keys, so whole slices of keys are masked."""
    gen = torch.Generator().manual_seed(seed)
    J = K - 1
    M = K * J
    block_of_mask = torch.arange(K).repeat_interleave(J)
    limit_offset = torch.cat((torch.arange(K), block_of_mask))
    allow_tail = torch.cat((torch.full((K,), -1), block_of_mask))[:, None] == block_of_mask[None, :]
    L, R = Lw + M, K + M - first_row
    q = torch.randn(B, R, H, D, generator=gen).to(torch.bfloat16)
    k_cache, v_cache = (torch.randn(8, L + 1, Hkv, D, generator=gen).to(torch.bfloat16) for _ in range(2))
    n = torch.randint(0, Lw - K, (B,), generator=gen)
    n[0] = 0
    allow_cache = torch.arange(Lw)[None, None] <= (n[:, None] + limit_offset[None])[..., None]
    allowed = torch.cat((allow_cache, allow_tail[None].expand(B, -1, -1)), dim=2)[:, None]
    padded = torch.full((B, 1, K + M, L + 4), float("-inf"), dtype=torch.bfloat16)
    padded[..., :L].masked_fill_(allowed, 0.0)
    return q, k_cache, v_cache, padded, L, first_row


def _rows(padded, L, first_row):
    """The mask as the engine passes it: a view with padded (16-byte aligned) rows."""
    return padded[..., :L][:, :, first_row:]


def _sdpa(q, k_cache, v_cache, mask, scale):
    """SDPA's memory-efficient kernel on the same bf16 inputs (the eager path of model/model.py:357-361);
    grouped key heads are repeated to the query heads first, which that kernel needs here."""
    B, L, G = q.shape[0], mask.shape[-1], q.shape[2] // k_cache.shape[2]
    keys, vals = (t[:B, :L].repeat_interleave(G, dim=2) for t in (k_cache, v_cache))
    with sdpa_kernel(SDPBackend.EFFICIENT_ATTENTION):
        return F.scaled_dot_product_attention(q.transpose(1, 2), keys.transpose(1, 2), vals.transpose(1, 2),
                                              attn_mask=mask, scale=scale).transpose(1, 2)


@pytest.mark.parametrize("B,first_row,H,Hkv,D,Lw", [
    (1, 0, 16, 4, 256, 512), (3, 0, 16, 4, 256, 1024),     # attention layers: G = 4, 64 rows per key head
    (2, 4, 32, 32, 128, 2048), (4, 4, 32, 32, 128, 512),   # delta layers' mask rows: G = 1, 12 rows
    (2, 4, 32, 32, 128, 104),                              # one split of 128 keys: written directly
])
def test_decode_attention_error_within_sdpa_bounds(B, first_row, H, Hkv, D, Lw):
    q, k_cache, v_cache, padded, L, first = _attention_case(B * 100 + Lw, B, first_row, H, Hkv, D, Lw)
    scale = D ** -0.5
    ref = oracle.decode_attention_f32(q, k_cache, v_cache, _rows(padded, L, first), scale)
    qd, kd, vd, md = q.cuda(), k_cache.cuda(), v_cache.cuda(), _rows(padded.cuda(), L, first)
    out = gdn.decode_attention(qd, kd, vd, md, scale)
    sdpa = _sdpa(qd, kd, vd, md, scale)
    err, sdpa_err = (out.float().cpu() - ref).abs(), (sdpa.float().cpu() - ref).abs()
    assert not out.isnan().any()
    assert err.mean() <= 1.25 * sdpa_err.mean(), (err.mean(), sdpa_err.mean())
    assert err.max() <= 2 * sdpa_err.max(), (err.max(), sdpa_err.max())


def test_decode_attention_golden_and_fully_masked_row(golden):
    c = golden("decode_attention")
    out = gdn.decode_attention(c["q"].cuda(), c["k_cache"].cuda(), c["v_cache"].cuda(), c["mask"].cuda(), c["scale"])
    assert (out.float().cpu() - c["o_f32"]).abs().max() < 2e-2
    assert torch.equal(out[0, 2].cpu(), torch.zeros_like(out[0, 2].cpu()))


def test_decode_attention_no_keys_gives_zeros():
    q = torch.randn(2, 3, 4, 128, device="cuda").to(torch.bfloat16)
    cache = torch.randn(2, 8, 4, 128, device="cuda").to(torch.bfloat16)
    mask = torch.zeros(2, 1, 3, 0, device="cuda", dtype=torch.bfloat16)
    assert torch.equal(gdn.decode_attention(q, cache, cache, mask, 0.1), torch.zeros_like(q))


def test_decode_attention_rejects_unsupported():
    q = torch.randn(1, 65, 4, 128, device="cuda").to(torch.bfloat16)  # 65 rows per key head
    cache = torch.randn(1, 8, 4, 128, device="cuda").to(torch.bfloat16)
    mask = torch.zeros(1, 1, 65, 8, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="at most 64 query rows"):
        gdn.decode_attention(q, cache, cache, mask, 0.1)


def test_attention_kernels_leave_no_device_error():
    from jeeves_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.load().gdn_device_error(None, 0) == 0


@pytest.mark.parametrize("B,first_row,H,Hkv,D,Lw,K", [
    (1, 0, 32, 32, 128, 512, 4),     # 16 rows: the last row count of the single-warp issue path
    (2, 12, 16, 4, 256, 512, 4),     # 16 rows (R = 4, G = 4) at D = 256
    (2, 8, 32, 32, 128, 512, 5),     # 17 rows: one row in warp 1
    (2, 8, 16, 16, 256, 640, 5),     # 17 rows at D = 256
    (2, 6, 16, 4, 128, 1024, 4),     # 40 rows (R = 10, G = 4): warp 2 partly filled
    (2, 6, 16, 4, 256, 1024, 4),     # 40 rows at D = 256
    (2, 5, 32, 16, 128, 512, 5),     # 40 rows (R = 20, G = 2)
])
def test_decode_attention_row_counts_around_the_warp_edges(B, first_row, H, Hkv, D, Lw, K):
    """Row counts that switch the issuing lane (16 / 17 rows) and leave a live warp past warp 0
    partly filled, at both head dims, held to the same SDPA-relative bounds."""
    q, k_cache, v_cache, padded, L, first = _attention_case(B * 77 + Lw + first_row, B, first_row, H, Hkv, D, Lw, K)
    scale = D ** -0.5
    ref = oracle.decode_attention_f32(q, k_cache, v_cache, _rows(padded, L, first), scale)
    qd, kd, vd, md = q.cuda(), k_cache.cuda(), v_cache.cuda(), _rows(padded.cuda(), L, first)
    out = gdn.decode_attention(qd, kd, vd, md, scale)
    sdpa = _sdpa(qd, kd, vd, md, scale)
    err, sdpa_err = (out.float().cpu() - ref).abs(), (sdpa.float().cpu() - ref).abs()
    assert not out.isnan().any()
    assert err.mean() <= 1.25 * sdpa_err.mean(), (err.mean(), sdpa_err.mean())
    assert err.max() <= 2 * sdpa_err.max(), (err.max(), sdpa_err.max())


@pytest.mark.parametrize("D,Lw", [(128, 2048), (128, 104), (256, 512)])
@pytest.mark.parametrize("poison", [float("nan"), float("inf")])
def test_decode_attention_ignores_cache_slots_past_the_keys(D, Lw, poison):
    """Cache slots at or past L (stale entries the engine may leave there) hold NaN or Inf: the
    output must stay finite and equal to the output with finite values in those slots, as the
    reference's masked loads (other=0) make it."""
    H = Hkv = 32 if D == 128 else 16
    q, k_cache, v_cache, padded, L, first = _attention_case(Lw + D, 2, 4, H, Hkv, D, Lw)
    tail = torch.randn(8, 40, Hkv, D).to(torch.bfloat16)
    k_clean, v_clean = torch.cat((k_cache, tail), 1), torch.cat((v_cache, tail), 1)
    k_bad, v_bad = k_clean.clone(), v_clean.clone()
    k_bad[:, L:] = poison
    v_bad[:, L:] = poison
    md = _rows(padded.cuda(), L, first)
    scale = D ** -0.5
    clean = gdn.decode_attention(q.cuda(), k_clean.cuda(), v_clean.cuda(), md, scale)
    bad = gdn.decode_attention(q.cuda(), k_bad.cuda(), v_bad.cuda(), md, scale)
    assert torch.isfinite(bad.float()).all()
    assert same_bits(bad, clean)
