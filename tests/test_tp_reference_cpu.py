"""The fp32 restatement behind the tensor-parallel parity checks
(TPLlamaDecoder.reference_logits: batched dense attention over the gathered
context) against a per-row, per-head loop of the same decode step, on the CPU
with a small model shape."""
import torch
import torch.nn.functional as F

from serving_engine_b200.tp_decode import TPConfig, TPLlamaDecoder

SMALL = TPConfig(layers=2, hidden=512, heads=8, kv_heads=4, head_dim=64, ffn=1024, vocab=1000)


def loop_reference(dec: TPLlamaDecoder, tokens: torch.Tensor) -> torch.Tensor:
    cfg, b, d = dec.cfg, dec.batch, dec.cfg.head_dim
    g = cfg.heads // cfg.kv_heads
    x = F.embedding(tokens, dec.embed).float()
    kv = dec.kv.float().clone()
    for li, w in enumerate(dec.layers):
        h = F.rms_norm(x, (cfg.hidden,), w["n1"].float(), cfg.eps)
        qkv = h @ w["wqkv"].float().t()
        q = dec._rope(qkv[:, :cfg.heads * d].view(b, cfg.heads, d), dec.cos.float(), dec.sin.float())
        k = dec._rope(qkv[:, cfg.heads * d:(cfg.heads + cfg.kv_heads) * d].view(b, cfg.kv_heads, d),
                      dec.cos.float(), dec.sin.float())
        v = qkv[:, (cfg.heads + cfg.kv_heads) * d:].view(b, cfg.kv_heads, d)
        kv[li, 0].view(-1, cfg.kv_heads, d)[dec.slots] = k.to(torch.bfloat16).float()
        kv[li, 1].view(-1, cfg.kv_heads, d)[dec.slots] = v.to(torch.bfloat16).float()
        o = torch.empty(b, cfg.heads, d)
        for r in range(b):
            blocks = dec.block_table[r].long()
            ks = kv[li, 0][blocks].reshape(-1, cfg.kv_heads, d)[:dec.context]
            vs = kv[li, 1][blocks].reshape(-1, cfg.kv_heads, d)[:dec.context]
            for hh in range(cfg.heads):
                o[r, hh] = torch.softmax((ks[:, hh // g] @ q[r, hh]) * dec.scale, dim=0) @ vs[:, hh // g]
        x = x + o.reshape(b, -1) @ w["wo"].float().t()
        h = F.rms_norm(x, (cfg.hidden,), w["n2"].float(), cfg.eps)
        gu = h @ w["wgu"].float().t()
        f = gu.shape[1] // 2
        x = x + (F.silu(gu[:, :f]) * gu[:, f:]) @ w["wd"].float().t()
    h = F.rms_norm(x, (cfg.hidden,), dec.final_norm.float(), cfg.eps)
    return h @ dec.lm_head.float().t()


def test_reference_logits_match_a_per_row_loop():
    dec = TPLlamaDecoder(SMALL, 0, 1, torch.device("cpu"), batch=3, context=70, seed=2)
    tokens = torch.tensor([5, 17, 900])
    kv_before = dec.kv.clone()
    ref = dec.reference_logits(tokens)
    assert torch.equal(dec.kv, kv_before)
    torch.testing.assert_close(ref, loop_reference(dec, tokens), atol=1e-5, rtol=1e-5)
