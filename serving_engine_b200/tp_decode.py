"""Tensor-parallel Llama decode step over the paged KV pool (one process per GPU).

The model and its KV block pool are sharded by KV head across the ranks of the
process group: rank r holds kv heads [r*H/N, (r+1)*H/N) and the query heads of
their GQA groups, the matching column slices of q/k/v and gate/up
(column-parallel) and row slices of o_proj and down_proj (row-parallel). The
only communication is an NCCL all-reduce(SUM) of the [batch, hidden] partial
sums after o_proj and after down_proj; attention runs on each rank's own pool
shard with this library's kernels (KV append, paged decode attention) and
needs no exchange. Embedding and lm_head are replicated.

Weights are random (seeded per full matrix, then sliced), so every TP degree
computes the same model. The decode step can be captured in a CUDA graph
(including the NCCL all-reduces) and replayed with new tokens.

With ``fused=True`` (the default) the layer glue runs as this library's kernels:
RoPE fused with the KV append, each residual add fused with the following
RMSNorm, and SwiGLU in one pass; ``fused=False`` runs the same math as eager
torch ops. With ``allreduce="peer"`` (fused only, world > 1) each all-reduce
and the residual add + RMSNorm after it are one kernel over CUDA IPC peer
memory (``PeerAllReduceNorm``) instead of NCCL followed by the add + norm
kernel: o_proj and down_proj write their partial sums straight into this
rank's peer buffer, and the residual stream lives there too.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import ops

BLOCK_SIZE = 16


@dataclass
class TPConfig:
    layers: int = 32
    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    vocab: int = 128256
    rope_theta: float = 500000.0
    eps: float = 1e-5


LLAMA3_8B = TPConfig()


def _full(shape, seed: int, device, std: float) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std).to(torch.bfloat16)


class TPLlamaDecoder:
    """Sharded Llama for batched decode at a fixed context (synthetic pre-filled KV)."""

    def __init__(self, cfg: TPConfig, rank: int, world: int, device, batch: int, context: int, seed: int = 0,
                 group=None, fill_kv: bool = True, fused: bool = True, allreduce: str = "nccl"):
        if cfg.kv_heads % world or cfg.heads % world or cfg.ffn % world:
            raise ValueError(f"{world} ranks must divide kv heads {cfg.kv_heads}, heads {cfg.heads}, ffn {cfg.ffn}")
        if allreduce not in ("nccl", "peer") or (allreduce == "peer" and not fused):
            raise ValueError(f"allreduce must be 'nccl' or 'peer' (peer needs fused=True), got {allreduce!r}")
        self.cfg, self.rank, self.world, self.device, self.group = cfg, rank, world, device, group
        self.fused = fused
        self.allreduce = allreduce if world > 1 else "nccl"  # one rank: nothing to reduce
        self.batch, self.context = batch, context
        hkv = cfg.kv_heads // world
        hq = cfg.heads // world
        d = cfg.head_dim
        self.hq, self.hkv = hq, hkv
        f_l = cfg.ffn // world
        std = 0.02
        self.embed = _full((cfg.vocab, cfg.hidden), seed * 7919 + 1, device, std)
        self.lm_head = _full((cfg.vocab, cfg.hidden), seed * 7919 + 2, device, std)
        self.final_norm = torch.ones(cfg.hidden, dtype=torch.bfloat16, device=device)
        self.layers = []
        q_rows = slice(rank * hq * d, (rank + 1) * hq * d)
        kv_rows = slice(rank * hkv * d, (rank + 1) * hkv * d)
        f_rows = slice(rank * f_l, (rank + 1) * f_l)
        for li in range(cfg.layers):
            s = seed * 7919 + 1000 * (li + 1)
            wq = _full((cfg.heads * d, cfg.hidden), s + 1, device, std)[q_rows]
            wk = _full((cfg.kv_heads * d, cfg.hidden), s + 2, device, std)[kv_rows]
            wv = _full((cfg.kv_heads * d, cfg.hidden), s + 3, device, std)[kv_rows]
            wo = _full((cfg.hidden, cfg.heads * d), s + 4, device, std)[:, q_rows]
            wg = _full((cfg.ffn, cfg.hidden), s + 5, device, std)[f_rows]
            wu = _full((cfg.ffn, cfg.hidden), s + 6, device, std)[f_rows]
            wd = _full((cfg.hidden, cfg.ffn), s + 7, device, std)[:, f_rows]
            self.layers.append({
                "wqkv": torch.cat([wq, wk, wv]).contiguous(),   # column-parallel
                "wo": wo.contiguous(),                           # row-parallel
                "wgu": torch.cat([wg, wu]).contiguous(),         # column-parallel
                "wd": wd.contiguous(),                           # row-parallel
                "n1": torch.ones(cfg.hidden, dtype=torch.bfloat16, device=device),
                "n2": torch.ones(cfg.hidden, dtype=torch.bfloat16, device=device),
            })
            del wq, wk, wv, wo, wg, wu, wd
        # KV pool shard: every sequence owns ceil(context / 16) blocks; the
        # current token is appended at position context - 1 each step.
        self.blocks_per_seq = math.ceil(context / BLOCK_SIZE)
        self.bps = (ops.decode_blocks_per_split(batch, hkv, self.blocks_per_seq, device)
                    if torch.device(device).type == "cuda" else 0)
        nb = batch * self.blocks_per_seq
        self.kv = torch.empty(cfg.layers, 2, nb, BLOCK_SIZE, hkv, d, dtype=torch.bfloat16, device=device)
        if fill_kv:
            for li in range(cfg.layers):
                for pl in range(2):
                    # the full (all kv heads) pool plane is seeded; this rank keeps its heads
                    g = torch.Generator(device=device).manual_seed(seed * 7919 + 500000 + 2 * li + pl)
                    full = torch.randn((nb, BLOCK_SIZE, cfg.kv_heads, d), generator=g, device=device,
                                       dtype=torch.float32)
                    self.kv[li, pl].copy_(full[:, :, rank * hkv:(rank + 1) * hkv].to(torch.bfloat16))
                    del full
        # fixed step metadata: row b owns blocks [b*bps, (b+1)*bps) (a shuffled permutation)
        g = torch.Generator().manual_seed(seed + 17)
        perm = torch.randperm(nb, generator=g).view(batch, self.blocks_per_seq).to(torch.int32)
        self.block_table = perm.to(device)
        self.q_starts = torch.arange(batch, dtype=torch.int32, device=device)
        self.k_lens = torch.full((batch,), context, dtype=torch.int32, device=device)
        self.q_pos = torch.full((batch,), context - 1, dtype=torch.int32, device=device)
        last_block = perm[:, (context - 1) // BLOCK_SIZE].to(torch.int64)
        self.slots = (last_block * BLOCK_SIZE + (context - 1) % BLOCK_SIZE).to(device)
        positions = torch.full((batch,), context - 1, dtype=torch.float32, device=device)
        inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, device=device, dtype=torch.float32) / d))
        ang = positions[:, None] * inv_freq[None, :]
        self.cos = torch.cat([ang.cos(), ang.cos()], dim=-1).to(torch.bfloat16)[:, None, :]
        self.sin = torch.cat([ang.sin(), ang.sin()], dim=-1).to(torch.bfloat16)[:, None, :]
        self.scale = 1.0 / math.sqrt(d)
        self.tokens = torch.zeros(batch, dtype=torch.int64, device=device)
        self.graph = None
        self.ar = None
        if self.allreduce == "peer":
            from .peer_allreduce import PeerAllReduceNorm

            self.ar = PeerAllReduceNorm(batch, cfg.hidden, torch.bfloat16, device, group)

    def _all_reduce(self, x: torch.Tensor) -> None:
        if self.world > 1:
            torch.distributed.all_reduce(x, group=self.group)

    @staticmethod
    def _rope(x, cos, sin):
        half = x.shape[-1] // 2
        rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
        return x * cos + rot * sin

    def mlp(self, h: torch.Tensor, w: dict) -> torch.Tensor:
        """SwiGLU with gate/up column-parallel and down row-parallel, then all-reduce."""
        gu = h @ w["wgu"].t()
        f_l = gu.shape[1] // 2
        dn = (F.silu(gu[:, :f_l]) * gu[:, f_l:]) @ w["wd"].t()
        self._all_reduce(dn)
        return dn

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        """One decode step for all sequences; returns the greedy next tokens."""
        return self.logits(tokens).argmax(dim=-1)

    def logits(self, tokens: torch.Tensor) -> torch.Tensor:
        if self.fused:
            return self._logits_fused(tokens)
        cfg, b, d = self.cfg, self.batch, self.cfg.head_dim
        x = F.embedding(tokens, self.embed)
        for li, w in enumerate(self.layers):
            h = F.rms_norm(x, (cfg.hidden,), w["n1"], cfg.eps)
            qkv = h @ w["wqkv"].t()
            q = qkv[:, :self.hq * d].view(b, self.hq, d)
            k = qkv[:, self.hq * d:(self.hq + self.hkv) * d].view(b, self.hkv, d)
            v = qkv[:, (self.hq + self.hkv) * d:].view(b, self.hkv, d)
            q = self._rope(q, self.cos, self.sin)
            k = self._rope(k, self.cos, self.sin)
            kc, vc = self.kv[li, 0], self.kv[li, 1]
            ops.kv_append(k, v, kc, vc, self.slots)
            o, _ = ops.paged_decode(q, kc, vc, self.block_table, self.q_starts, self.k_lens, self.q_pos, self.hq,
                                    self.hkv, self.scale, True, blocks_per_split=self.bps)
            a = o.view(b, self.hq * d) @ w["wo"].t()
            self._all_reduce(a)
            x = x + a
            x = x + self.mlp(F.rms_norm(x, (cfg.hidden,), w["n2"], cfg.eps), w)
        h = F.rms_norm(x, (cfg.hidden,), self.final_norm, cfg.eps)
        return h @ self.lm_head.t()

    def _logits_fused(self, tokens: torch.Tensor) -> torch.Tensor:
        """The decode step with the fused layer kernels (same math as the eager path)."""
        if self.ar is not None:
            return self._logits_peer(tokens)
        cfg, b, d = self.cfg, self.batch, self.cfg.head_dim
        x = F.embedding(tokens, self.embed)  # residual stream, updated in place
        h = ops.add_rmsnorm(x, None, self.layers[0]["n1"], cfg.eps)
        for li, w in enumerate(self.layers):
            qkv = h @ w["wqkv"].t()
            kc, vc = self.kv[li, 0], self.kv[li, 1]
            q = ops.rope_kv_append(qkv, self.cos, self.sin, self.slots, kc, vc, self.hq, self.hkv)
            o, _ = ops.paged_decode(q, kc, vc, self.block_table, self.q_starts, self.k_lens, self.q_pos, self.hq,
                                    self.hkv, self.scale, True, blocks_per_split=self.bps)
            a = o.view(b, self.hq * d) @ w["wo"].t()
            self._all_reduce(a)
            h = ops.add_rmsnorm(x, a, w["n2"], cfg.eps)
            dn = ops.swiglu(h @ w["wgu"].t()) @ w["wd"].t()
            self._all_reduce(dn)
            nxt = self.layers[li + 1]["n1"] if li + 1 < len(self.layers) else self.final_norm
            h = ops.add_rmsnorm(x, dn, nxt, cfg.eps)
        return h @ self.lm_head.t()

    def _logits_peer(self, tokens: torch.Tensor) -> torch.Tensor:
        """The fused decode step with each all-reduce + add + RMSNorm as one
        peer-memory kernel; the residual stream is ``self.ar.x``."""
        cfg, b, d, ar = self.cfg, self.batch, self.cfg.head_dim, self.ar
        torch.index_select(self.embed, 0, tokens, out=ar.x)
        h = ops.add_rmsnorm(ar.x, None, self.layers[0]["n1"], cfg.eps)
        for li, w in enumerate(self.layers):
            qkv = h @ w["wqkv"].t()
            kc, vc = self.kv[li, 0], self.kv[li, 1]
            q = ops.rope_kv_append(qkv, self.cos, self.sin, self.slots, kc, vc, self.hq, self.hkv)
            o, _ = ops.paged_decode(q, kc, vc, self.block_table, self.q_starts, self.k_lens, self.q_pos, self.hq,
                                    self.hkv, self.scale, True, blocks_per_split=self.bps)
            torch.mm(o.view(b, self.hq * d), w["wo"].t(), out=ar.partial)
            h = ar(w["n2"], cfg.eps)
            torch.mm(ops.swiglu(h @ w["wgu"].t()), w["wd"].t(), out=ar.partial)
            nxt = self.layers[li + 1]["n1"] if li + 1 < len(self.layers) else self.final_norm
            h = ar(nxt, cfg.eps)
        return h @ self.lm_head.t()

    @torch.inference_mode()
    def reference_logits(self, tokens: torch.Tensor) -> torch.Tensor:
        """The same decode step in fp32 with dense attention over each row's
        gathered context, for an unsharded decoder (world 1: it holds every
        weight and kv head). The new token's K/V (rounded to the pool's bf16) is
        written to a copy of the pool at the row's slot, as the step writes it;
        the decoder's own pool is left untouched."""
        if self.world != 1:
            raise ValueError("reference_logits needs the unsharded (world 1) decoder")
        cfg, b, d = self.cfg, self.batch, self.cfg.head_dim
        g = cfg.heads // cfg.kv_heads
        x = F.embedding(tokens, self.embed).float()
        cos, sin = self.cos.float(), self.sin.float()
        for li, w in enumerate(self.layers):
            h = F.rms_norm(x, (cfg.hidden,), w["n1"].float(), cfg.eps)
            qkv = h @ w["wqkv"].float().t()
            q = self._rope(qkv[:, :cfg.heads * d].view(b, cfg.heads, d), cos, sin)
            k = self._rope(qkv[:, cfg.heads * d:(cfg.heads + cfg.kv_heads) * d].view(b, cfg.kv_heads, d), cos, sin)
            v = qkv[:, (cfg.heads + cfg.kv_heads) * d:].view(b, cfg.kv_heads, d)
            kc = self.kv[li, 0].float().view(-1, cfg.kv_heads, d)
            vc = self.kv[li, 1].float().view(-1, cfg.kv_heads, d)
            kc[self.slots] = k.to(torch.bfloat16).float()
            vc[self.slots] = v.to(torch.bfloat16).float()
            slots = (self.block_table.long()[:, :, None] * BLOCK_SIZE
                     + torch.arange(BLOCK_SIZE, device=x.device)).view(b, -1)[:, :self.context]
            ks, vs = kc[slots], vc[slots]  # [b, context, kv heads, d]
            ks = ks.repeat_interleave(g, dim=2)
            vs = vs.repeat_interleave(g, dim=2)
            sc = torch.einsum("bhd,bthd->bht", q, ks) * self.scale
            o = torch.einsum("bht,bthd->bhd", torch.softmax(sc, dim=-1), vs)
            x = x + o.reshape(b, -1) @ w["wo"].float().t()
            h = F.rms_norm(x, (cfg.hidden,), w["n2"].float(), cfg.eps)
            gu = h @ w["wgu"].float().t()
            f = gu.shape[1] // 2
            x = x + (F.silu(gu[:, :f]) * gu[:, f:]) @ w["wd"].float().t()
        h = F.rms_norm(x, (cfg.hidden,), self.final_norm.float(), cfg.eps)
        return h @ self.lm_head.float().t()

    def capture(self, warmup: int = 2) -> None:
        """Record one decode step into a CUDA graph (after eager warm-up steps)."""
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self.tokens.copy_(self.forward(self.tokens))
        torch.cuda.current_stream(self.device).wait_stream(s)
        # workspace and error word exist before capture; capture allocates nothing else outside the graph pool
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out_tokens = self.forward(self.tokens)

    def step(self) -> None:
        """Replay (or run) one decode step; the greedy tokens feed the next step."""
        if self.graph is not None:
            self.graph.replay()
            self.tokens.copy_(self.out_tokens)
        else:
            self.tokens.copy_(self.forward(self.tokens))

    def release(self) -> None:
        """Drop the CUDA graph (it holds NCCL work) and the peer buffers
        (collective) before the process group goes away."""
        self.graph = None
        self.out_tokens = None
        if self.ar is not None:
            self.ar.close()
            self.ar = None
