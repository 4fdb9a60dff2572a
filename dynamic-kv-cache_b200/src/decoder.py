"""Random-init Llama-style text decoder of the SmolLM2-360M shape.

The reference runs the pretrained SmolVLM2 text model (HF LlamaModel) and routes
its attention through GPUCache (src/gpu_cache.py:151-183); the checkpoint is not
part of this build, so this module restates the decoder itself with random
weights: 32 layers, hidden 960, 15 query / 5 KV heads of dim 64, SiLU MLP of
width 2560, RMSNorm eps 1e-5, rotary embeddings (theta 100000), tied embeddings,
bf16. Projections use the joined QKV and gate/up weights of the reference's fused
mode (src/gpu_ops.py:26-47). With a GPUCache the attention is the packed-KV path
(append + attend on the sm_100a kernels); with a NativeCache it is plain bf16
history + SDPA (the reference's "native" mode).
"""
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import gpu_kernels as K
from .gpu_cache import GPUCache, RequestBatch, append_many, attend_many
from .gpu_ops import activation_product, add_rms, cuda_rms


@dataclass(frozen=True)
class DecoderConfig:
    layers: int = 32
    hidden: int = 960
    q_heads: int = 15
    kv_heads: int = 5
    head_dim: int = 64
    intermediate: int = 2560
    vocab: int = 49280
    rms_eps: float = 1e-5
    rope_theta: float = 100000.0
    init_std: float = 0.02


SMOLLM2_360M = DecoderConfig()


class NativeCache:
    """Unquantised bf16 history per layer (the reference's native DynamicCache mode)."""

    def __init__(self, layers):
        self.k = [None] * layers
        self.v = [None] * layers

    def get_seq_length(self, layer_idx=0):
        return 0 if self.k[layer_idx] is None else self.k[layer_idx].shape[2]

    def update(self, k, v, layer):
        self.k[layer] = k if self.k[layer] is None else torch.cat((self.k[layer], k), 2)
        self.v[layer] = v if self.v[layer] is None else torch.cat((self.v[layer], v), 2)
        return self.k[layer], self.v[layer]

    def fork(self):
        other = NativeCache(len(self.k))
        other.k, other.v = list(self.k), list(self.v)  # torch.cat never mutates: sharing is safe
        return other


def rope_tables(cfg, positions, device):
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, cfg.head_dim, 2, device=device, dtype=torch.float32) / cfg.head_dim))
    freqs = positions.float()[:, None] * inv[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos(), emb.sin()


def apply_rope(x, cos, sin):
    """HF Llama rotate-half rotary embedding over the last dimension (computed in
    fp32; cos / sin broadcast against x)."""
    half = x.shape[-1] // 2
    xf = x.float()
    rot = torch.cat((-xf[..., half:], xf[..., :half]), dim=-1)
    return (xf * cos + rot * sin).to(x.dtype)


class Decoder(torch.nn.Module):
    def __init__(self, cfg=SMOLLM2_360M, device='cuda', dtype=torch.bfloat16, seed=0):
        super().__init__()
        self.cfg = cfg
        gen = torch.Generator(device='cpu').manual_seed(seed)

        def w(*shape):
            return torch.nn.Parameter((torch.randn(*shape, generator=gen) * cfg.init_std).to(dtype).to(device),
                                      requires_grad=False)

        qkv_out = (cfg.q_heads + 2 * cfg.kv_heads) * cfg.head_dim
        self.embed = w(cfg.vocab, cfg.hidden)
        self.qkv = torch.nn.ParameterList([w(qkv_out, cfg.hidden) for _ in range(cfg.layers)])
        self.o = torch.nn.ParameterList([w(cfg.hidden, cfg.q_heads * cfg.head_dim) for _ in range(cfg.layers)])
        self.gate_up = torch.nn.ParameterList([w(2 * cfg.intermediate, cfg.hidden) for _ in range(cfg.layers)])
        self.down = torch.nn.ParameterList([w(cfg.hidden, cfg.intermediate) for _ in range(cfg.layers)])
        ones = lambda: torch.nn.Parameter(torch.ones(cfg.hidden, dtype=dtype, device=device), requires_grad=False)
        self.norm_attn = torch.nn.ParameterList([ones() for _ in range(cfg.layers)])
        self.norm_mlp = torch.nn.ParameterList([ones() for _ in range(cfg.layers)])
        self.norm_out = ones()

    def rms(self, x, weight):
        return cuda_rms(x, weight, self.cfg.rms_eps)

    def add_norm(self, x, y, weight):
        """(x + y, its RMSNorm * weight): the residual add and the next norm of a
        layer in one call (one launch on CUDA); y None: (x, norm of x)."""
        return add_rms(x, y, weight, self.cfg.rms_eps)

    def run_layers(self, x, attend):
        """The decoder layers over x: attend(h, layer) is a layer's attention of the
        normed input h, o_proj included. Returns the last residual stream."""
        c = self.cfg
        x, h = self.add_norm(x, None, self.norm_attn[0])
        for layer in range(c.layers):
            x, h = self.add_norm(x, attend(h, layer), self.norm_mlp[layer])
            gate, up = F.linear(h, self.gate_up[layer]).chunk(2, dim=-1)
            m = F.linear(activation_product(gate, up), self.down[layer])
            if layer + 1 < c.layers:
                x, h = self.add_norm(x, m, self.norm_attn[layer + 1])
            else:
                x = x + m
        return x

    def project_qkv(self, x, layer, cos, sin):
        """q [B, q_heads, n, d] and k / v [B, kv_heads, n, d] of x [B, n, hidden]: one
        joined projection and one rotary pass over the query and key heads together
        (cos / sin [B or 1, n, 1, d]); q, k and v are strided views, which the cache
        kernels take as they are."""
        c = self.cfg
        b, n = x.shape[0], x.shape[1]
        h = F.linear(x, self.qkv[layer]).view(b, n, c.q_heads + 2 * c.kv_heads, c.head_dim)
        if h.is_cuda:  # one launch, bit-identical to apply_rope
            qk = K.rotary(h, cos, sin, c.q_heads + c.kv_heads)
        else:  # the native-cache decoder on the CPU
            qk = apply_rope(h[:, :, :c.q_heads + c.kv_heads], cos, sin)
        q = qk[:, :, :c.q_heads].transpose(1, 2)
        k = qk[:, :, c.q_heads:].transpose(1, 2)
        v = h[:, :, c.q_heads + c.kv_heads:].transpose(1, 2)
        return q, k, v

    def rotary(self, positions, b, n, device):
        """cos / sin [b, n, 1, d] of positions [b * n] (or [n] for b = 1)."""
        cos, sin = rope_tables(self.cfg, positions.reshape(-1), device)
        return cos.view(b, n, 1, -1), sin.view(b, n, 1, -1)

    def attention(self, x, layer, cache, cos, sin):
        n = x.shape[1]
        q, k, v = self.project_qkv(x, layer, cos, sin)
        if isinstance(cache, GPUCache):
            out = cache.append_attend(q, k, v, layer)  # append + attend in one call; [1, n, q_heads, d]
        else:
            past = cache.get_seq_length(layer)
            kk, vv = cache.update(k, v, layer)
            mask = torch.arange(past + n, device=x.device)[None, :] <= past + torch.arange(n, device=x.device)[:, None]
            out = F.scaled_dot_product_attention(q, kk, vv, attn_mask=mask, enable_gqa=True).transpose(1, 2)
        return F.linear(out.reshape(1, n, -1), self.o[layer])

    def attention_chunks(self, x, layer, cache, cos, sin):
        """Attention of B token chunks x [B, n, hidden] side by side over the cache's
        history: each chunk sees the history and its own earlier tokens; nothing is
        appended (the packed path runs one batched kernel call per layer)."""
        b, n = x.shape[0], x.shape[1]
        q, k, v = self.project_qkv(x, layer, cos, sin)
        past = cache.get_seq_length(layer)
        if isinstance(cache, GPUCache):
            out = cache.attend_batched(q, k, v, layer, past)  # [B, n, q_heads, d]
        else:
            if past:
                k = torch.cat((cache.k[layer].expand(b, -1, -1, -1), k), 2)
                v = torch.cat((cache.v[layer].expand(b, -1, -1, -1), v), 2)
            mask = torch.arange(past + n, device=x.device)[None, :] <= past + torch.arange(n, device=x.device)[:, None]
            out = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, enable_gqa=True).transpose(1, 2)
        return F.linear(out.reshape(b, n, -1), self.o[layer])

    def attention_many(self, x, layer, caches, cos, sin):
        """Attention of B requests' frames x [B, n, hidden], request r over caches[r],
        appending each frame's K/V to its own cache (one pack and one attention
        launch for all of them)."""
        b, n = x.shape[0], x.shape[1]
        q, k, v = self.project_qkv(x, layer, cos, sin)
        pasts = append_many(caches, k, v, layer)
        out = attend_many(caches, q, k, v, layer, pasts)  # [B, n, q_heads, d]
        return F.linear(out.reshape(b, n, -1), self.o[layer])

    def forward_many(self, caches, ids=None, embeds=None, logits=0):
        """forward() for B independent requests stepped together (request batching,
        not in the reference): ids [B, n] or embeds [B, n, hidden], request r appended
        to caches[r] (GPUCache objects with their own pools; their histories may
        differ in length). Returns fp32 logits [B, logits, vocab] (or None)."""
        x = self.embed[ids] if embeds is None else embeds
        b, n = x.shape[0], x.shape[1]
        if len(caches) != b:
            raise ValueError('one cache per request')
        pasts = torch.tensor([c.get_seq_length(0) for c in caches], device=x.device)
        positions = pasts[:, None] + torch.arange(n, device=x.device)[None, :]  # [B, n]
        cos, sin = self.rotary(positions, b, n, x.device)
        x = self.run_layers(x, lambda h, layer: self.attention_many(h, layer, caches, cos, sin))
        if not logits:
            return None
        h = self.rms(x[:, -logits:], self.norm_out)
        return F.linear(h, self.embed).float()

    def forward_device(self, batch, x, logits=0):
        """One frame step of the B requests of `batch` (a RequestBatch whose
        prepare() has run): x [B, n, hidden]. Like forward_many, but every cache
        operation reads the batch's device-resident descriptors, so the whole step
        can be captured once as a CUDA graph and replayed (FrameGraph)."""
        c = self.cfg
        b, n = x.shape[0], x.shape[1]
        cos, sin = self.rotary(batch.positions, b, n, x.device)

        def attend(h, layer):
            q, k, v = self.project_qkv(h, layer, cos, sin)
            out = torch.empty((b, n, c.q_heads, c.head_dim), dtype=h.dtype, device=h.device)
            if batch.append:
                K.append_attention_many_device(q, k, v, batch.targets_ptr, batch.histories_ptr, b, batch.max_past,
                                               out, layer, n, c.kv_heads, c.q_heads // c.kv_heads, c.head_dim,
                                               c.layers)
            else:
                K.packed_attention_many_device(q, k, v, batch.histories_ptr, b, batch.max_past, out, layer, n,
                                               c.kv_heads, c.q_heads // c.kv_heads, c.head_dim, c.layers)
            return F.linear(out.reshape(b, n, -1), self.o[layer])

        x = self.run_layers(x, attend)
        if not logits:
            return None
        h = self.rms(x[:, -logits:], self.norm_out)
        return F.linear(h, self.embed).float()

    def forward_chunks(self, cache, ids, logits):
        """B equal-length token chunks (ids [B, n]) after the cache's history, side by
        side, without appending; returns fp32 logits [B, logits, vocab] of each
        chunk's last `logits` positions."""
        x = self.embed[ids]
        n = x.shape[1]
        past = cache.get_seq_length(0)
        cos, sin = self.rotary(torch.arange(past, past + n, device=x.device), 1, n, x.device)
        x = self.run_layers(x, lambda h, layer: self.attention_chunks(h, layer, cache, cos, sin))
        h = self.rms(x[:, -logits:], self.norm_out)
        return F.linear(h, self.embed).float()

    def forward(self, cache, ids=None, embeds=None, logits=0):
        """Runs n new tokens (ids [1, n] or embeds [1, n, hidden]) through every layer,
        appending their K/V to `cache`; returns fp32 logits of the last `logits`
        positions (or None)."""
        x = self.embed[ids] if embeds is None else embeds
        n = x.shape[1]
        past = cache.get_seq_length(0)
        cos, sin = self.rotary(torch.arange(past, past + n, device=x.device), 1, n, x.device)
        x = self.run_layers(x, lambda h, layer: self.attention(h, layer, cache, cos, sin))
        if not logits:
            return None
        h = self.rms(x[:, -logits:], self.norm_out)
        return F.linear(h, self.embed).float()


class FrameGraph:
    """Frame steps of B requests replayed from one CUDA graph (the graph-captured
    append of every layer; not in the reference, which launches each layer's
    kernels from Python on every frame). The first step runs eagerly (it is also
    the warm-up); the graph of the whole decoder step is then captured once and
    every later step is: host bookkeeping + one descriptor copy (RequestBatch),
    one input copy, one graph replay. Steps must keep the frame length n; the
    caches' precision may change per step (select() before step()). With
    append=False the steps attend over the caches' histories without appending
    (query chunks side by side, e.g. candidates over one fork)."""

    def __init__(self, model, caches, n, logits=0, max_past=None, append=True):
        self.model, self.n, self.logits = model, n, logits
        self.batch = RequestBatch(caches, n, max_past, append)
        dev = self.batch.device
        self.x = torch.empty((len(caches), n, model.cfg.hidden), dtype=model.embed.dtype, device=dev)
        self.stream = torch.cuda.Stream(dev)
        self.graph = None
        self.out = None

    def rebind(self, caches):
        """Serves another set of caches (same count and geometry) with the same
        captured graph: the next steps append to them."""
        self.batch.rebind(caches)

    def step(self, embeds=None, ids=None):
        """Appends one frame (embeds [B, n, hidden] or ids [B, n]) to every cache;
        returns the logits of the last `logits` positions (None if 0). The returned
        tensor is the graph's output buffer: the next step overwrites it."""
        x = self.model.embed[ids] if embeds is None else embeds
        if tuple(x.shape) != tuple(self.x.shape):
            raise ValueError(f'frame step expects inputs of shape {tuple(self.x.shape)}')
        self.batch.prepare()
        self.x.copy_(x)
        if self.graph is not None:
            self.graph.replay()
            return self.out
        current = torch.cuda.current_stream(self.batch.device)
        self.stream.wait_stream(current)
        with torch.cuda.stream(self.stream):
            out = self.model.forward_device(self.batch, self.x, self.logits)  # the eager first step (warm-up)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=self.stream):
                self.out = self.model.forward_device(self.batch, self.x, self.logits)
        current.wait_stream(self.stream)
        self.graph = graph
        return out
