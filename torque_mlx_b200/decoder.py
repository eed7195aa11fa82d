"""Random-init GQA decoder whose attention runs on the packed rotated KV cache
(benchmark config 5: the model around the packed-KV path).

A plain pre-norm decoder (RMSNorm, RoPE, SwiGLU MLP, bf16 weights drawn from
N(0, 0.02)) with one ``TorqueKVCache`` per layer.  In the token step the
projections run as this library's one-token GEMV (tq_gemv, with RMSNorm /
SwiGLU / fp32-input prologues), RoPE as tq_rope_qk; the dense prefill uses
torch ops.  The KV path is this library too: prompt
tokens are packed in bulk after a dense causal prefill, each generated token
is packed and attended straight on the packed codes in one fused call
(tq_decode_append).  The whole per-token step can be captured in one CUDA graph.

Rotation folding (reference: src/torque_mlx/conversion.py:19-51 and the Qwen
adapter's runtime rotation, families/qwen.py:521-528, qwen_mlx.py:758-760):

* ``fold="full"``: Pi folded into W_Q, W_K, W_V and Pi^T into W_O, as benchmark
  config 5 specifies.  RoPE then acts on rotated q/k, which is a different
  (self-consistent) model from the unfolded one, since Pi and RoPE do not
  commute; for random weights that is immaterial.
* ``fold="vo_only"``: Pi folded into W_V / W_O only; q and k are rotated at run
  time after RoPE by the append / decode kernels, which reproduces the
  unfolded model exactly (up to quantization).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import ops
from .cache import TorqueKVCache
from .config import TorqueConfig
from .rotation import RotationSpec


@dataclass(frozen=True)
class DecoderConfig:
    num_layers: int = 28
    hidden: int = 2048
    q_heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 6144
    vocab: int = 151936
    bits: int = 4
    rope_theta: float = 1_000_000.0
    rms_eps: float = 1e-6
    init_std: float = 0.02
    fold: str = "full"  # "full" | "vo_only"
    seed: int = 0
    rotation_seed: int = 0


class PackedKVDecoder:
    def __init__(self, cfg: DecoderConfig, *, max_tokens: int = 4096, device: torch.device | str = "cuda",
                 decode_mode: str = "auto"):
        if cfg.fold not in ("full", "vo_only"):
            raise ValueError("fold must be 'full' or 'vo_only'")
        self.cfg = cfg
        self.dev = torch.device(device)
        g = torch.Generator(device=self.dev)
        g.manual_seed(cfg.seed)
        bf = torch.bfloat16
        H, Hkv, d, D = cfg.q_heads, cfg.kv_heads, cfg.head_dim, cfg.hidden

        def w(*shape):
            return (torch.randn(shape, generator=g, device=self.dev, dtype=torch.float32) * cfg.init_std).to(bf)

        self.rotation = RotationSpec.from_seed(head_dim=d, seed=cfg.rotation_seed)
        self.embed = w(cfg.vocab, D)
        self.lm_head = w(cfg.vocab, D)
        self.final_norm = torch.ones(D, device=self.dev, dtype=bf)
        self.layers = []
        for _ in range(cfg.num_layers):
            wq, wk, wv, wo = w(H * d, D), w(Hkv * d, D), w(Hkv * d, D), w(D, H * d)
            if cfg.fold == "full":
                wq, wk = self._rotate_out_rows(wq, H), self._rotate_out_rows(wk, Hkv)
            wv = self._rotate_out_rows(wv, Hkv)
            wo = self._rotate_in_cols(wo, H)
            self.layers.append(dict(
                attn_norm=torch.ones(D, device=self.dev, dtype=bf), mlp_norm=torch.ones(D, device=self.dev, dtype=bf),
                wqkv=torch.cat([wq, wk, wv], 0).contiguous(), wo=wo.contiguous(),
                w_gate_up=torch.cat([w(cfg.ffn, D), w(cfg.ffn, D)], 0).contiguous(), w_down=w(D, cfg.ffn)))
        full = cfg.fold == "full"
        kv_cfg = TorqueConfig(bit_width=cfg.bits, head_dim=d, num_layers=1, kv_heads=Hkv, fused_weights=True,
                              rotation_seed=cfg.rotation_seed)
        self.caches = [TorqueKVCache(config=kv_cfg, initial_capacity=max_tokens, decode_mode=decode_mode,
                                     rotate_keys_on_append=not full, rotate_values_on_append=False,
                                     rotate_queries_on_decode=not full) for _ in range(cfg.num_layers)]
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, device=self.dev, dtype=torch.float32) / d))
        ang = torch.arange(max_tokens + 1, device=self.dev, dtype=torch.float32)[:, None] * inv[None]
        self.cos, self.sin = ang.cos(), ang.sin()  # [pos, d/2]
        self.pos = torch.zeros((), dtype=torch.long, device=self.dev)  # next position (device, for graphs)
        self._qf = torch.empty((cfg.q_heads, d), dtype=torch.float32, device=self.dev)  # roped q of the step
        self._kr = torch.empty((cfg.kv_heads, d), dtype=bf, device=self.dev)         # roped k of the step
        self.length = 0
        self.graph = None

    # -- weight folding: Pi acts on each head's d-block -------------------------
    def _rotate_out_rows(self, wmat: torch.Tensor, heads: int) -> torch.Tensor:
        """W' = Pi W per head block of output rows (columns of a block are rotated)."""
        d = self.cfg.head_dim
        blocks = wmat.float().reshape(heads, d, -1).transpose(1, 2).contiguous()  # [h, in, d]
        return self.rotation.apply(blocks).transpose(1, 2).reshape(heads * d, -1).to(wmat.dtype)

    def _rotate_in_cols(self, wmat: torch.Tensor, heads: int) -> torch.Tensor:
        """W' = W Pi^T per head block of input columns (rows of a block are rotated)."""
        d = self.cfg.head_dim
        blocks = wmat.float().reshape(-1, heads, d).contiguous()
        return self.rotation.apply(blocks).reshape(wmat.shape).to(wmat.dtype)

    # -- pieces ---------------------------------------------------------------------
    def _rms(self, x, weight):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.cfg.rms_eps)).to(x.dtype) * weight

    def _rope(self, x, cos, sin):
        """x [..., T, d] with cos/sin [T, d/2] (rotate-half convention)."""
        x1, x2 = x[..., ::2].float(), x[..., 1::2].float()
        out = torch.stack([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1).flatten(-2)
        return out.to(x.dtype)

    def _mlp(self, x, lay):
        gu = x @ lay["w_gate_up"].T
        gate, up = gu.chunk(2, dim=-1)
        return (F.silu(gate) * up) @ lay["w_down"].T

    # -- prefill --------------------------------------------------------------------
    @torch.no_grad()
    def prefill(self, tokens: torch.Tensor) -> torch.Tensor:
        """Dense causal attention over the prompt, then pack every layer's K/V
        into its cache in one append.  Returns the last position's logits."""
        cfg = self.cfg
        T = int(tokens.numel())
        H, Hkv, d = cfg.q_heads, cfg.kv_heads, cfg.head_dim
        x = self.embed[tokens.to(self.dev)]
        cos, sin = self.cos[self.length:self.length + T], self.sin[self.length:self.length + T]
        for lay, cache in zip(self.layers, self.caches):
            h = self._rms(x, lay["attn_norm"])
            qkv = h @ lay["wqkv"].T
            q, k, v = qkv.split([H * d, Hkv * d, Hkv * d], dim=-1)
            q = self._rope(q.reshape(T, H, d).transpose(0, 1), cos, sin)
            k = self._rope(k.reshape(T, Hkv, d).transpose(0, 1), cos, sin)
            v = v.reshape(T, Hkv, d).transpose(0, 1)
            # (in vo_only mode the cache rotates q and k; scores are invariant under that rotation)
            att = F.scaled_dot_product_attention(q[None], k[None], v[None], is_causal=True, enable_gqa=True)[0]
            x = x + att.transpose(0, 1).reshape(T, H * d) @ lay["wo"].T
            x = x + self._mlp(self._rms(x, lay["mlp_norm"]), lay)
            cache.append(key=k.contiguous(), value=v.contiguous())  # [Hkv, T, d]
        self.length += T
        self.pos.fill_(self.length)
        return self._rms(x[-1:], self.final_norm) @ self.lm_head.T

    # -- one generated token --------------------------------------------------------
    def _step_body(self, token: torch.Tensor, captured: bool) -> torch.Tensor:
        """One token through every layer in seven launches a layer:
        tq_gemv (RMSNorm fused) for qkv, tq_rope_qk, the fused packed-KV step
        (decode kernel packing the token + split merge), tq_gemv for the
        output projection with the residual, tq_gemv (RMSNorm fused) for
        gate/up and tq_gemv (SwiGLU fused) for down with the residual."""
        cfg = self.cfg
        H, Hkv, d = cfg.q_heads, cfg.kv_heads, cfg.head_dim
        # index_select keeps the lookup on the device (graph-safe, no host sync)
        x = torch.index_select(self.embed, 0, token.reshape(1)).reshape(-1)
        qf, kr = self._qf, self._kr
        for lay, cache in zip(self.layers, self.caches):
            qkv = ops.gemv(lay["wqkv"], x, mode="rms", norm_weight=lay["attn_norm"], eps=cfg.rms_eps)
            ops.rope_qk(qkv, self.cos, self.sin, self.pos, H, Hkv, d, qf, kr)
            v = qkv[(H + Hkv) * d:]
            if captured:
                # one fused launch packs the token and attends (tq_decode_append)
                att = cache._step(kr.reshape(1, 1, Hkv, 1, d), v.reshape(1, 1, Hkv, 1, d), qf, H,
                                  advance=True, return_lse=False, full_capacity=True)[0]
            else:
                att = cache.append_decode(key=kr, value=v.reshape(Hkv, d), query=qf)
            x = ops.gemv(lay["wo"], att.reshape(-1), mode="f32", residual=x)
            gu = ops.gemv(lay["w_gate_up"], x, mode="rms", norm_weight=lay["mlp_norm"], eps=cfg.rms_eps)
            x = ops.gemv(lay["w_down"], gu, mode="silu", residual=x)
        self.pos.add_(1)
        return ops.gemv(self.lm_head, x, mode="rms", norm_weight=self.final_norm, eps=cfg.rms_eps).reshape(1, -1)

    @torch.no_grad()
    def step(self, token: torch.Tensor) -> torch.Tensor:
        """Eager decode of one token (reference-facing path); returns logits [1, vocab]."""
        logits = self._step_body(token.to(self.dev), captured=False)
        self.length += 1
        return logits

    @torch.no_grad()
    def capture(self) -> None:
        """Capture the whole per-token step (all layers) in one CUDA graph."""
        self._tok = torch.zeros((), dtype=torch.long, device=self.dev)
        side = torch.cuda.Stream(device=self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(side):
            # size every cache's workspace for the capacity plan before capture
            for cache in self.caches:
                cache._decode(torch.zeros((self.cfg.q_heads, self.cfg.head_dim), device=self.dev), self.cfg.q_heads,
                              extra=0, return_lse=False, full_capacity=True)
            side.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=side):
                self._logits = self._step_body(self._tok, captured=True)
                self._next = self._logits.argmax(-1).reshape(())
        torch.cuda.current_stream(self.dev).wait_stream(side)

    @torch.no_grad()
    def step_graph(self, token: torch.Tensor) -> torch.Tensor:
        """Replay the captured step for ``token`` (device scalar); returns the
        greedy next token (device scalar) and leaves logits in ``self._logits``."""
        if self.graph is None:
            self.capture()
        if self.length + 1 > self.caches[0].capacity:
            raise RuntimeError("cache capacity reached")
        self._tok.copy_(token.reshape(()))
        self.graph.replay()
        for cache in self.caches:
            cache._len_host += 1
        self.length += 1
        return self._next

    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, new_tokens: int, *, use_graph: bool = True) -> torch.Tensor:
        logits = self.prefill(prompt)
        tok = logits.argmax(-1).reshape(())
        out = [tok]
        for _ in range(new_tokens - 1):
            if use_graph:
                tok = self.step_graph(tok).clone()
            else:
                tok = self.step(tok).argmax(-1).reshape(())
            out.append(tok)
        return torch.stack(out)
