"""Decode-layer fusions of the tensor-parallel decoder, through the C ABI:
RoPE + KV append bit-identical to the eager tensor ops followed by the KV
write, residual add + RMSNorm and SwiGLU against fp32 torch (one rounding of
the 16-bit output: within an ulp), and the fused decode step against the eager
one."""
import math

import pytest
import torch
import torch.nn.functional as F

from serving_engine_b200 import check_device_errors, ops
from serving_engine_b200.tp_decode import TPConfig, TPLlamaDecoder

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rope_eager(x, cos, sin):
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos + rot * sin


def rope_tables(pos, d, dtype):
    inv = 1.0 / (10000.0 ** (torch.arange(0, d, 2, device=DEV, dtype=torch.float32) / d))
    ang = pos.float()[:, None] * inv[None, :]
    return (torch.cat([ang.cos(), ang.cos()], -1).to(dtype)[:, None, :],
            torch.cat([ang.sin(), ang.sin()], -1).to(dtype)[:, None, :])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hq,hkv,d", [(32, 8, 128), (8, 8, 64), (16, 2, 128), (32, 8, 64)])
# 0: contiguous rows take the 16-byte-vector kernel; 2: a row stride of w + 2
# elements the element-pair path; 1: a 2-byte-offset view the element-at-a-time path
@pytest.mark.parametrize("offset", [0, 2, 1])
def test_rope_kv_append_bit_exact(dtype, hq, hkv, d, offset):
    g = torch.Generator(device=DEV).manual_seed(hq * d + offset)
    n, nb = 37, 20
    w = (hq + 2 * hkv) * d
    if offset == 0:
        qkv = torch.randn(n, w, generator=g, device=DEV).to(dtype)
    else:
        qkv = torch.randn(n, w + 2, generator=g, device=DEV).to(dtype)[:, offset % 2:offset % 2 + w]
    pos = torch.randint(0, 4000, (n,), generator=g, device=DEV)
    cos, sin = rope_tables(pos, d, dtype)
    slots = torch.randperm(nb * 16, generator=g, device=DEV)[:n]
    kc = torch.randn(nb, 16, hkv, d, generator=g, device=DEV).to(dtype)
    vc = torch.randn(nb, 16, hkv, d, generator=g, device=DEV).to(dtype)
    kc_ref, vc_ref = kc.clone(), vc.clone()
    q = ops.rope_kv_append(qkv, cos, sin, slots, kc, vc, hq, hkv)
    torch.cuda.synchronize()
    check_device_errors()
    q_ref = rope_eager(qkv[:, :hq * d].view(n, hq, d), cos, sin)
    k_ref = rope_eager(qkv[:, hq * d:(hq + hkv) * d].view(n, hkv, d), cos, sin)
    v_ref = qkv[:, (hq + hkv) * d:].view(n, hkv, d)
    kc_ref.view(-1, hkv, d)[slots] = k_ref
    vc_ref.view(-1, hkv, d)[slots] = v_ref
    assert torch.equal(q, q_ref)
    assert torch.equal(kc, kc_ref)
    assert torch.equal(vc, vc_ref)


@pytest.mark.parametrize("pad", [0, 2])  # 0: the 16-byte-vector kernel; 2: the warp-per-row kernel
def test_rope_kv_append_bad_slot_sets_error_and_skips(pad):
    hq, hkv, d, nb = 4, 2, 64, 4
    qkv = torch.randn(3, (hq + 2 * hkv) * d + pad, device=DEV).to(torch.bfloat16)[:, :(hq + 2 * hkv) * d]
    cos, sin = rope_tables(torch.tensor([1, 2, 3], device=DEV), d, torch.bfloat16)
    kc = torch.zeros(nb, 16, hkv, d, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.tensor([0, nb * 16, 5], device=DEV)  # the middle one is out of range
    ops.rope_kv_append(qkv, cos, sin, slots, kc, vc, hq, hkv)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="slot"):
        check_device_errors()
    assert kc.view(-1, hkv, d)[0].abs().sum() > 0 and kc.view(-1, hkv, d)[5].abs().sum() > 0
    assert vc.view(-1, hkv, d)[[1, 2, 3, 4, 6]].abs().sum() == 0


def assert_within_ulp(out, ref32):
    """One rounding of the 16-bit output away from the fp32 result."""
    sig = 8 if out.dtype == torch.bfloat16 else 11
    ulp = torch.exp2(torch.floor(torch.log2(ref32.abs().clamp_min(1e-30))) - (sig - 1))
    assert bool(((out.float() - ref32).abs() <= ulp + 1e-6).all()), float((out.float() - ref32).abs().max())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n,hidden", [(256, 4096), (3, 2048), (5, 10000), (4, 1001)])
def test_add_rmsnorm(dtype, n, hidden):
    g = torch.Generator(device=DEV).manual_seed(hidden + n)
    x = torch.randn(n, hidden, generator=g, device=DEV).to(dtype)
    a = torch.randn(n, hidden, generator=g, device=DEV).to(dtype)
    w = (1 + 0.1 * torch.randn(hidden, generator=g, device=DEV)).to(dtype)
    x_ref = x + a
    out = ops.add_rmsnorm(x, a, w, 1e-5)
    torch.cuda.synchronize()
    assert torch.equal(x, x_ref)  # the residual stream is the eager bf16 sum
    xf = x_ref.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5) * w.float()
    assert_within_ulp(out, ref)
    out2 = ops.add_rmsnorm(x, None, w, 1e-5)  # no residual: x unchanged
    assert torch.equal(x, x_ref)
    assert_within_ulp(out2, ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("ffn", [1792, 1001])  # 1001: the element-at-a-time path
def test_swiglu(dtype, ffn):
    g = torch.Generator(device=DEV).manual_seed(3)
    gu = (2 * torch.randn(77, 2 * ffn, generator=g, device=DEV)).to(dtype)
    out = ops.swiglu(gu)
    torch.cuda.synchronize()
    f = gu.shape[1] // 2
    ref = F.silu(gu[:, :f].float()) * gu[:, f:].float()
    # silu's exponential is the fast hardware one: allow one more ulp of slack
    sig = 8 if dtype == torch.bfloat16 else 11
    ulp = torch.exp2(torch.floor(torch.log2(ref.abs().clamp_min(1e-30))) - (sig - 1))
    assert bool(((out.float() - ref).abs() <= 2 * ulp + 1e-5).all())


def test_fused_tp_step_matches_eager():
    cfg = TPConfig(layers=2, hidden=512, heads=8, kv_heads=4, head_dim=64, ffn=1024, vocab=1000)
    tokens = torch.randint(0, cfg.vocab, (6,), generator=torch.Generator().manual_seed(1)).cuda()
    out = {}
    for fused in (False, True):
        dec = TPLlamaDecoder(cfg, 0, 1, torch.device(DEV), batch=6, context=300, seed=2, fused=fused)
        out[fused] = dec.logits(tokens).float()
        check_device_errors()
    cos = F.cosine_similarity(out[True], out[False], dim=-1)
    assert float(cos.min()) > 0.9999, cos
    assert torch.equal(out[True].argmax(-1), out[False].argmax(-1))
    assert math.isfinite(float(out[True].abs().max()))
