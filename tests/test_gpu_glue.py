"""Decoder glue kernels (tq_rmsnorm / tq_rope_qk / tq_silu_mul) against the
PyTorch ops they replace, and one decoder step built from them against the
same step written with PyTorch ops (bf16 model; tolerances stated per test)."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

from torque_mlx_b200 import ops  # noqa: E402
from torque_mlx_b200.decoder import DecoderConfig, PackedKVDecoder  # noqa: E402


def _torch_rms(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


def _torch_rope(x, cos, sin):
    x1, x2 = x[..., ::2].float(), x[..., 1::2].float()
    return torch.stack([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1).flatten(-2).to(x.dtype)


def _bf16_close(got, want, frac_exact=0.98):
    """Equal up to one bf16 rounding step, and mostly bit-equal."""
    got, want = got.float(), want.float()
    tol = want.abs() * 2.0 ** -7 + 1e-6
    assert bool(((got - want).abs() <= tol).all()), float((got - want).abs().max())
    assert float((got == want).float().mean()) >= frac_exact


@pytest.mark.parametrize("rows,n", [(1, 2048), (5, 256), (3, 6144)])
def test_rmsnorm_matches_torch(rows, n):
    g = torch.Generator(device="cuda").manual_seed(n + rows)
    x = (torch.randn(rows, n, generator=g, device="cuda") * 3).to(torch.bfloat16)
    w = (torch.rand(n, generator=g, device="cuda") + 0.5).to(torch.bfloat16)
    _bf16_close(ops.rmsnorm(x, w, 1e-6), _torch_rms(x, w, 1e-6))


@pytest.mark.parametrize("hq,hkv,d", [(16, 8, 128), (4, 2, 64), (16, 2, 256)])
def test_rope_qk_matches_torch(hq, hkv, d):
    g = torch.Generator(device="cuda").manual_seed(d)
    qkv = torch.randn(1, (hq + 2 * hkv) * d, generator=g, device="cuda").to(torch.bfloat16)
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2, device="cuda", dtype=torch.float32) / d))
    ang = torch.arange(64, device="cuda", dtype=torch.float32)[:, None] * inv[None]
    cos, sin = ang.cos(), ang.sin()
    pos = torch.tensor(37, device="cuda")
    q_out = torch.empty(hq, d, device="cuda")
    k_out = torch.empty(hkv, d, device="cuda", dtype=torch.bfloat16)
    ops.rope_qk(qkv, cos, sin, pos, hq, hkv, d, q_out, k_out)
    q, k, _ = qkv.split([hq * d, hkv * d, hkv * d], dim=-1)
    c, s = cos[37:38], sin[37:38]
    # same op sequence and roundings: bit-equal
    assert torch.equal(q_out, _torch_rope(q.reshape(hq, 1, d), c, s).reshape(hq, d).float())
    assert torch.equal(k_out, _torch_rope(k.reshape(hkv, 1, d), c, s).reshape(hkv, d))


@pytest.mark.parametrize("rows,f", [(1, 6144), (4, 512)])
def test_silu_mul_matches_torch(rows, f):
    g = torch.Generator(device="cuda").manual_seed(f)
    gu = (torch.randn(rows, 2 * f, generator=g, device="cuda") * 2).to(torch.bfloat16)
    gate, up = gu.chunk(2, dim=-1)
    _bf16_close(ops.silu_mul(gu), F.silu(gate) * up)


def test_glue_step_matches_torch_step():
    """Logits of a decoder step built from the glue kernels and the fused
    packed-KV step equal (to bf16 noise) the same step written with PyTorch
    ops and separate append / decode calls."""
    cfg = DecoderConfig(num_layers=2, hidden=256, q_heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1000, bits=4,
                        seed=9)
    a = PackedKVDecoder(cfg, max_tokens=256)
    b = PackedKVDecoder(cfg, max_tokens=256)
    prompt = torch.randint(0, cfg.vocab, (40,), generator=torch.Generator().manual_seed(3)).cuda()
    a.prefill(prompt)
    b.prefill(prompt)
    H, Hkv, d = cfg.q_heads, cfg.kv_heads, cfg.head_dim
    tok = torch.tensor(17, device="cuda")
    for _ in range(3):
        got = a.step(tok).float()
        x = b.embed[tok.reshape(1)]
        cos, sin = b.cos[b.length:b.length + 1], b.sin[b.length:b.length + 1]
        for lay, cache in zip(b.layers, b.caches):
            qkv = _torch_rms(x, lay["attn_norm"], cfg.rms_eps) @ lay["wqkv"].T
            q, k, v = qkv.split([H * d, Hkv * d, Hkv * d], dim=-1)
            q = _torch_rope(q.reshape(H, 1, d), cos, sin).reshape(H, d)
            k = _torch_rope(k.reshape(Hkv, 1, d), cos, sin).reshape(Hkv, d)
            cache.append(key=k, value=v.reshape(Hkv, d))
            att = cache.decode(query=q.float())
            x = x + att.reshape(1, H * d).to(x.dtype) @ lay["wo"].T
            gate, up = (_torch_rms(x, lay["mlp_norm"], cfg.rms_eps) @ lay["w_gate_up"].T).chunk(2, dim=-1)
            x = x + (F.silu(gate) * up) @ lay["w_down"].T
        b.length += 1
        b.pos.add_(1)
        want = (_torch_rms(x, b.final_norm, cfg.rms_eps) @ b.lm_head.T).float()
        scale = float(want.abs().max())
        assert float((got - want).abs().max()) <= 0.03 * scale, (float((got - want).abs().max()), scale)
        tok = want.argmax(-1).reshape(())


@pytest.mark.parametrize("mode", ["bf16", "f32", "rms", "silu"])
@pytest.mark.parametrize("n,k", [(2048, 2048), (4096, 2048), (2048, 6144), (1000, 256), (3, 512)])
@pytest.mark.parametrize("res", [False, True])
def test_gemv_matches_fp32_reference(mode, n, k, res):
    """tq_gemv against W x' in float64 over the same bf16 x' (the prologue
    output the PyTorch ops produce); one bf16 rounding of an fp32 sum."""
    g = torch.Generator(device="cuda").manual_seed(n + k)
    w = (torch.randn(n, k, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    nw = (torch.rand(k, generator=g, device="cuda") + 0.5).to(torch.bfloat16)
    if mode == "silu":
        x = torch.randn(2 * k, generator=g, device="cuda").to(torch.bfloat16)
        xp = ops.silu_mul(x.reshape(1, -1)).reshape(-1)
    elif mode == "f32":
        x = torch.randn(k, generator=g, device="cuda")
        xp = x.to(torch.bfloat16)
    elif mode == "rms":
        x = torch.randn(k, generator=g, device="cuda").to(torch.bfloat16)
        xp = ops.rmsnorm(x.reshape(1, -1), nw, 1e-6).reshape(-1)
    else:
        x = torch.randn(k, generator=g, device="cuda").to(torch.bfloat16)
        xp = x
    r = torch.randn(n, generator=g, device="cuda").to(torch.bfloat16) if res else None
    got = ops.gemv(w, x, mode=mode, norm_weight=nw, eps=1e-6, residual=r).double()
    want = w.double() @ xp.double() + (r.double() if res else 0)
    tol = 2.0 ** -7 * want.abs() + 1e-3
    assert bool(((got - want).abs() <= tol).all()), float((got - want).abs().max())
