"""Batched greedy decoding over a Hugging Face Llama-3 / Qwen2 / Qwen2.5 / Qwen3
model with this package's KV caches and decode attention (the reference's
Engine, exactkv/engine.py:18-103: same constructor, prefill / step / generate /
kv_bytes and the same hooks).

The model's own modules do everything except the cache and the decode
attention, so an engine on CompressedKV and one on BF16KV compute identical
logits (the compressed cache is lossless and the two attention kernels are
bit-identical). Prefill runs the model's forward pass one sequence at a time
and encodes its keys/values straight from the model's [1, H, T, D] cache
layout (strided reads, no transposed copy); all sequences share one prompt
length (as in the reference).
"""
import torch

from .attention import decode_attention
from .cache import BF16KV, CompressedKV, check_overflow
from .kernels import P

BACKENDS = {"exactkv": CompressedKV, "bf16": BF16KV}
_SUPPORTED = ("llama", "qwen2", "qwen3")


def _rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def _rope(x, cos, sin):
    """x [B, H, 1, D]; cos, sin [B or 1, 1, D] from the model's rotary embedding."""
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    return x * cos + _rotate_half(x) * sin


class Engine:
    def __init__(self, model, B, T_max, backend="exactkv", attn=None, before_step=None):
        """model: a loaded HF causal LM (Llama-3, Qwen2/2.5, Qwen3; head dim 128,
        no sliding window). backend: 'exactkv', 'bf16' or a cache class with the
        same interface. attn(q, k_cache, v_cache) replaces decode_attention;
        before_step(engine, T) runs before each step (benchmark hooks)."""
        cfg = model.config
        if cfg.model_type not in _SUPPORTED:
            raise ValueError(f"supported model types: {_SUPPORTED} (got {cfg.model_type})")
        if getattr(cfg, "use_sliding_window", False):
            raise ValueError("sliding-window attention is not supported")
        self.m = model
        self.L = cfg.num_hidden_layers
        self.Hq, self.Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
        self.D = getattr(cfg, "head_dim", None) or cfg.hidden_size // self.Hq
        if self.D != 128:
            raise ValueError("head dim 128 only")
        self.B = B
        self.TS = -(-T_max // P) * P
        cache = BACKENDS.get(backend, backend)
        dev = next(model.parameters()).device
        self.kv = [(cache(B, self.TS, self.Hkv, self.D, device=dev), cache(B, self.TS, self.Hkv, self.D, device=dev))
                   for _ in range(self.L)]
        self.attn = attn or decode_attention
        self.before_step = before_step
        self.qk_norm = hasattr(model.model.layers[0].self_attn, "k_norm")   # Qwen3
        self.grows = 0

    @property
    def T(self):
        return self.kv[0][0].T

    @staticmethod
    def _layer_kv(pkv, i):
        """Keys and values [1, Hkv, T, D] of layer i from an HF cache object."""
        if hasattr(pkv, "layers"):
            return pkv.layers[i].keys, pkv.layers[i].values
        return pkv.key_cache[i], pkv.value_cache[i]

    def _logits(self, h):
        return self.m.lm_head(self.m.model.norm(h))

    @torch.no_grad()
    def prefill(self, ids):
        """ids: [B, T] token ids. Returns each sequence's greedy next token, [B]."""
        nxt = torch.empty(ids.shape[0], dtype=torch.long, device=ids.device)
        for b in range(ids.shape[0]):
            out = self.m.model(ids[b:b + 1], use_cache=True)
            for i, (kc, vc) in enumerate(self.kv):
                k, v = self._layer_kv(out.past_key_values, i)
                # the encoder reads the HF layout [1, H, T, D] through strides: no transposed copy
                kc.prefill_slot(b, k.transpose(1, 2))
                vc.prefill_slot(b, v.transpose(1, 2))
            nxt[b] = self._logits(out.last_hidden_state[:, -1]).argmax(-1)[0]
            del out
        return nxt

    def _attend(self, i, layer, x, cos, sin):
        """Self-attention of layer i for one new token per sequence; x [B, 1, hidden]."""
        att, B, D = layer.self_attn, self.B, self.D
        q = att.q_proj(x).view(B, 1, self.Hq, D)
        k = att.k_proj(x).view(B, 1, self.Hkv, D)
        v = att.v_proj(x).view(B, 1, self.Hkv, D)
        if self.qk_norm:
            q, k = att.q_norm(q), att.k_norm(k)
        q = _rope(q.transpose(1, 2), cos, sin)            # [B, Hq, 1, D]
        k = _rope(k.transpose(1, 2), cos, sin)            # [B, Hkv, 1, D]
        kc, vc = self.kv[i]
        kc.append(k[:, :, 0])
        vc.append(v[:, 0])
        o = self.attn(q[:, :, 0].contiguous(), kc, vc)    # [B, Hq, D]
        return att.o_proj(o.reshape(B, 1, self.Hq * D))

    @torch.no_grad()
    def step(self, tok):
        """tok: [B] current tokens. Returns bf16 logits [B, vocab] of the next token."""
        m, T = self.m, self.T
        if self.before_step:
            self.before_step(self, T + 1)
        h = m.model.embed_tokens(tok.view(self.B, 1))
        cos, sin = m.model.rotary_emb(h, torch.full((1, 1), T, device=h.device))
        for i, layer in enumerate(m.model.layers):
            h = h + self._attend(i, layer, layer.input_layernorm(h), cos, sin)
            h = h + layer.mlp(layer.post_attention_layernorm(h))
        if (T + 1) % P == 0:
            self.grows += check_overflow([c for pair in self.kv for c in pair])
        return self._logits(h)[:, 0]

    @torch.no_grad()
    def generate(self, ids, n_new):
        """Greedy decoding: (tokens [B, n_new], logits [B, n_new - 1, vocab])."""
        t = self.prefill(ids)
        toks, logits = [t], []
        for _ in range(n_new - 1):
            lg = self.step(t)
            logits.append(lg)
            t = lg.argmax(-1)
            toks.append(t)
        return torch.stack(toks, 1), torch.stack(logits, 1)

    def kv_bytes(self):
        return sum(c.nbytes() for pair in self.kv for c in pair)
