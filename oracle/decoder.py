"""TEST INFRASTRUCTURE ONLY — fp32 CPU restatement of the streaming decoder path.

Llama-style decoder (RMSNorm, rotate-half rotary embeddings, GQA, SiLU MLP, tied
embeddings) whose attention follows the reference's CPU cache semantics
(src/cache_manager.py:43-63): every earlier segment is dequantised with unpack,
the current chunk stays native, attention runs over the concatenation; after a
frame's forward its K/V (rounded to bf16, the dtype the GPU path packs) are packed
with the frame's precision (src/kv_quantization.py:41-77). Candidate scoring
follows src/streaming.py:214-224: question + candidate on a copy of the video
history, mean (and sum) of the candidate tokens' log-likelihoods.
Weights are taken from the product decoder's parameters (same values), upcast to
fp32. The arithmetic is fp32, but every tensor the reference model holds in
bf16 (norm outputs, projection outputs, rotary output, attention output,
residual stream, logits — HF Llama in bf16, src/streaming.py:144-153) is rounded
to bf16 at the same point, so the K/V this oracle quantises are the values the
bf16 model would store.
"""
import numpy as np
import torch
import torch.nn.functional as F

from . import cpu_path, kvq


def _bits(t):
    return t.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)


def _bf(x):
    """Round fp32 values to bf16 (round-to-nearest-even) and back."""
    return x.to(torch.bfloat16).float()


class OracleDecoder:
    def __init__(self, cfg, params, memo=False):
        """params: dict name -> tensor (embed, qkv[i], o[i], gate_up[i], down[i],
        norm_attn[i], norm_mlp[i], norm_out), any dtype/device. memo=True keeps
        each stored segment's unpacked values after its first use (parity tests at
        full model shape); the timed CPU baseline leaves it off and unpacks the
        whole history on every call, as the reference does."""
        self.cfg = cfg
        self.memo = memo
        self.p = {k: v.detach().float().cpu() for k, v in params.items()}

    def _rms(self, x, w):
        return _bf(_bf(x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.cfg.rms_eps)) * w)

    def _rope(self, positions):
        c = self.cfg
        inv = 1.0 / (c.rope_theta ** (torch.arange(0, c.head_dim, 2, dtype=torch.float32) / c.head_dim))
        f = positions.float()[:, None] * inv[None, :]
        e = torch.cat((f, f), dim=-1)
        return e.cos(), e.sin()

    @staticmethod
    def _rot(x, cos, sin):
        h = x.shape[-1] // 2
        return x * cos + torch.cat((-x[..., h:], x[..., :h]), -1) * sin

    def forward(self, history, x, past, store_bits=None, logits=0):
        """history: per layer list of (K Packed, V Packed) segments. x: [1, n, hidden]
        fp32 embeddings. Appends this chunk packed with `store_bits` when given."""
        c = self.cfg
        n = x.shape[1]
        cos, sin = self._rope(torch.arange(past, past + n))
        for layer in range(c.layers):
            h = self._rms(x, self.p[f'norm_attn.{layer}'])
            q, k, v = _bf(F.linear(h, self.p[f'qkv.{layer}'])).split(
                [c.q_heads * c.head_dim, c.kv_heads * c.head_dim, c.kv_heads * c.head_dim], -1)
            q = _bf(self._rot(q.view(1, n, c.q_heads, c.head_dim).transpose(1, 2), cos, sin))
            k = _bf(self._rot(k.view(1, n, c.kv_heads, c.head_dim).transpose(1, 2), cos, sin))
            v = v.view(1, n, c.kv_heads, c.head_dim).transpose(1, 2)
            out = _bf(cpu_path.cpu_cache_attention(history[layer], q, k, v, memo=self.memo))  # [1, n, q_heads, d]
            if store_bits is not None:
                history[layer].append((kvq.pack(_bits(k), store_bits), kvq.pack(_bits(v), store_bits)))
            x = _bf(x + _bf(F.linear(out.reshape(1, n, -1), self.p[f'o.{layer}'])))
            h = self._rms(x, self.p[f'norm_mlp.{layer}'])
            gate, up = _bf(F.linear(h, self.p[f'gate_up.{layer}'])).chunk(2, -1)
            x = _bf(x + _bf(F.linear(_bf(_bf(F.silu(gate)) * up), self.p[f'down.{layer}'])))
        if not logits:
            return None
        return _bf(F.linear(self._rms(x[:, -logits:], self.p['norm_out']), self.p['embed']))

    def request(self, prefix_ids, frames, bits, question_ids, candidate_ids):
        """Prefix (16-bit), frames at their precision, then candidate scoring.
        Returns (mean log-likelihoods, summed log-likelihoods)."""
        emb = self.p['embed']
        history = [[] for _ in range(self.cfg.layers)]
        past = 0
        x = emb[prefix_ids[0].cpu()][None]
        self.forward(history, x, past, store_bits=16)
        past += x.shape[1]
        for f, b in zip(frames, bits):
            self.forward(history, f.float().cpu(), past, store_bits=b)
            past += f.shape[1]
        means, sums = [], []
        for cand in candidate_ids:
            ids = torch.cat((question_ids, cand), 1)[0].cpu()
            logits = self.forward([list(h) for h in history], emb[ids][None], past, logits=cand.shape[1] + 1)
            ll = logits[0, :-1].log_softmax(-1).gather(1, cand[0].cpu()[:, None])[:, 0]
            means.append(float(ll.mean()))
            sums.append(float(ll.sum()))
        return means, sums


def decoder_params(model):
    """Flattened parameter dict of the product Decoder (names as OracleDecoder expects)."""
    return {name: p for name, p in model.named_parameters()}
