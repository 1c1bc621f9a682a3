"""Batched greedy decoding over a Hugging Face Llama-3 / Qwen2 / Qwen2.5 / Qwen3
model with this package's KV caches (the reference's Engine interface,
exactkv/engine.py:18-103: constructor, prefill, step, generate, kv_bytes and the
attn / before_step hooks).

The model's own modules do everything except the cache and the decode
attention, so an engine on CompressedKV and one on BF16KV compute identical
logits: the compressed cache is lossless and the two attention kernels are
bit-identical.

Decode steps run from a CUDA graph. The token count lives on the device (one
int32 for the caches, one int64 for the rotary position), so one captured step
serves every step: the appends write at the device length, the attention
reads it (exk_attention_*_devlen), and the step ends by advancing it. The host
syncs once per `check_pages` pages to keep every compressed raw pool that many
worst-case pages ahead (CompressedKV.ensure_headroom) and captures again when
a pool had to move. With an attn or before_step hook, or graphs=False, the same
step runs eagerly.

Prefill runs the model's forward pass one sequence at a time and encodes its
keys/values straight from the model's [1, H, T, D] cache layout (strided reads,
no transposed copy); all sequences share one prompt length.
"""
import torch

from . import kernels
from .attention import decode_attention
from .cache import BF16KV, CompressedKV
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
    def __init__(self, model, B, T_max, backend="exactkv", attn=None, before_step=None, graphs=True,
                 check_pages=2, cache_kwargs=None):
        """model: a loaded HF causal LM (Llama-3, Qwen2/2.5, Qwen3; head dim 128,
        no sliding window). backend: 'exactkv', 'bf16' or a cache class with the
        same interface. attn(q, k_cache, v_cache) replaces decode_attention;
        before_step(engine, T) runs before each step (benchmark hooks; either
        one turns the CUDA graph off). cache_kwargs: extra arguments of the
        compressed caches (e.g. reserve)."""
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
        self.dev = next(model.parameters()).device
        kw = dict(cache_kwargs or {}) if cache is CompressedKV else {}
        self.kv = [(cache(B, self.TS, self.Hkv, self.D, device=self.dev, **kw),
                    cache(B, self.TS, self.Hkv, self.D, device=self.dev, **kw)) for _ in range(self.L)]
        self.compressed = isinstance(self.kv[0][0], CompressedKV)
        self.attn = attn
        self.before_step = before_step
        # hooks or a foreign cache class: host-side lengths, eager steps
        self._hooked = attn is not None or before_step is not None or cache not in (CompressedKV, BF16KV)
        self.graphs = graphs and not self._hooked
        self.check_pages = check_pages
        self.qk_norm = hasattr(model.model.layers[0].self_attn, "k_norm")   # Qwen3
        self.grows = 0
        self.captures = 0
        # step state on the device (inputs and outputs of the captured step)
        self._len = torch.zeros(1, dtype=torch.int32, device=self.dev)    # tokens held before the step
        self._pos = torch.zeros(1, dtype=torch.int64, device=self.dev)    # the same, as the rotary position
        self._tok = torch.zeros(B, dtype=torch.long, device=self.dev)
        self._logits = None
        self._next = torch.zeros(B, dtype=torch.long, device=self.dev)
        self._graph = None
        self._warmed = False
        self._next_check = 0

    @property
    def T(self):
        return self.kv[0][0].T

    def caches(self):
        return [c for pair in self.kv for c in pair]

    @staticmethod
    def _layer_kv(pkv, i):
        """Keys and values [1, Hkv, T, D] of layer i from an HF cache object."""
        if hasattr(pkv, "layers"):
            return pkv.layers[i].keys, pkv.layers[i].values
        return pkv.key_cache[i], pkv.value_cache[i]

    def _head(self, h):
        return self.m.lm_head(self.m.model.norm(h))

    # ------------------------------------------------------------------ prefill
    @torch.no_grad()
    def prefill(self, ids):
        """ids: [B, T] token ids. Returns each sequence's greedy next token, [B]."""
        first = torch.empty(ids.shape[0], dtype=torch.long, device=ids.device)
        for b in range(ids.shape[0]):
            out = self.m.model(ids[b:b + 1], use_cache=True)
            for i, (kc, vc) in enumerate(self.kv):
                k, v = self._layer_kv(out.past_key_values, i)
                # the encoder reads the HF layout [1, H, T, D] through strides: no transposed copy
                kc.prefill_slot(b, k.transpose(1, 2))
                vc.prefill_slot(b, v.transpose(1, 2))
            first[b] = self._head(out.last_hidden_state[:, -1]).argmax(-1)[0]
            del out
        self.sync_length()
        return first

    def sync_length(self):
        """Points the device-side length at the caches' host-side T (after a prefill
        or any host-side cache edit); the next graphed step captures again."""
        self._len.fill_(self.T)
        self._pos.fill_(self.T)
        self._graph = None
        self._next_check = self.T

    # ------------------------------------------------------------------ one decode step
    def _attend(self, i, layer, x, cos, sin):
        """Self-attention of layer i for one new token per sequence at the device
        length; x [B, 1, hidden]."""
        att, B, D = layer.self_attn, self.B, self.D
        q = att.q_proj(x).view(B, 1, self.Hq, D)
        k = att.k_proj(x).view(B, 1, self.Hkv, D)
        v = att.v_proj(x).view(B, 1, self.Hkv, D)
        if self.qk_norm:
            q, k = att.q_norm(q), att.k_norm(k)
        q = _rope(q.transpose(1, 2), cos, sin)[:, :, 0].contiguous()        # [B, Hq, D]
        k = _rope(k.transpose(1, 2), cos, sin)[:, :, 0]                      # [B, Hkv, D]
        v = v[:, 0]
        kc, vc = self.kv[i]
        if self._hooked:
            kc.append(k)
            vc.append(v)
            o = (self.attn or decode_attention)(q, kc, vc)
        elif self.compressed:
            kernels.append_token(k.contiguous(), kc, self._len)
            kernels.append_token(v.contiguous(), vc, self._len)
            o = kernels.attention_compressed_devlen(q, kc, vc, self._len, 1)
        else:
            kc.buf.index_copy_(1, self._pos, k.unsqueeze(1))
            vc.buf.index_copy_(1, self._pos, v.unsqueeze(1))
            o = kernels.attention_reference_devlen(q, kc.buf, vc.buf, self._len, 1)
        return att.o_proj(o.reshape(B, 1, self.Hq * D))

    def _body(self):
        """One decode step, enqueued on the current stream: reads self._tok and the
        device length, writes self._logits and self._next, advances the length."""
        m = self.m
        h = m.model.embed_tokens(self._tok.view(self.B, 1))
        cos, sin = m.model.rotary_emb(h, self._pos.view(1, 1))
        for i, layer in enumerate(m.model.layers):
            h = h + self._attend(i, layer, layer.input_layernorm(h), cos, sin)
            h = h + layer.mlp(layer.post_attention_layernorm(h))
        logits = self._head(h)[:, 0]
        if self._logits is None or self._logits.shape != logits.shape:
            self._logits = torch.empty_like(logits)
        self._logits.copy_(logits)
        torch.argmax(logits, -1, out=self._next)
        kernels.advance_length(self._len, 1)
        self._pos.add_(1)

    def _headroom(self):
        """One sync for every compressed cache: keep check_pages + 1 worst-case pages
        free. True when a pool moved."""
        cs = [c for c in self.caches() if isinstance(c, CompressedKV)]
        if not cs:
            return False
        used = torch.cat([c.cnt for c in cs] + [kernels.status_tensor(self.dev)]).tolist()
        if used[-1] != 0:
            kernels.check_status(self.dev)
        moved = [c._make_room(n, self.check_pages + 1) for c, n in zip(cs, used[:-1])]
        self.grows += sum(moved)
        return any(moved)

    def _note_step(self):
        for c in self.caches():
            if isinstance(c, CompressedKV):
                c.note_appended(1)
            else:
                c.T += 1

    @torch.no_grad()
    def _run(self, tok):
        """Runs one step for tokens `tok` (the graph when enabled); the outputs are
        left in self._logits and self._next."""
        if self.T >= self.TS:
            raise RuntimeError("the caches are full")
        if self.before_step:
            self.before_step(self, self.T + 1)
        self._tok.copy_(tok.view(-1))
        if self._hooked:
            self._eager_hooked()
            return
        if self.T >= self._next_check:
            if self._headroom():
                self._graph = None
            self._next_check = (self.T // P + self.check_pages) * P
        if not self.graphs or self._graph is None and not self._warmed:
            # eager: graphs off, or the first step, which warms cuBLAS and the
            # kernels' workspaces before the next step is captured
            self._warmed = True
            self._body()
            self._note_step()
            return
        if self._graph is None:
            torch.cuda.synchronize(self.dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._body()
            self._graph = g
            self.captures += 1
        self._graph.replay()
        self._note_step()

    def _eager_hooked(self):
        """The step with host-side lengths (hooks or a foreign cache class)."""
        m, T = self.m, self.T
        h = m.model.embed_tokens(self._tok.view(self.B, 1))
        cos, sin = m.model.rotary_emb(h, torch.full((1, 1), T, device=h.device))
        for i, layer in enumerate(m.model.layers):
            h = h + self._attend(i, layer, layer.input_layernorm(h), cos, sin)
            h = h + layer.mlp(layer.post_attention_layernorm(h))
        logits = self._head(h)[:, 0]
        self._logits = logits
        self._next = logits.argmax(-1)
        if self.T % P == 0:
            from .cache import check_overflow
            self.grows += check_overflow(self.caches())
        self._len.fill_(self.T)
        self._pos.fill_(self.T)

    @torch.no_grad()
    def step(self, tok):
        """tok: [B] current tokens. Returns bf16 logits [B, vocab] of the next token."""
        self._run(tok)
        return self._logits.clone()

    @torch.no_grad()
    def step_greedy(self, tok):
        """One step that returns only the greedy next tokens [B] (on the device; no
        logits copy)."""
        self._run(tok)
        return self._next.clone()

    @torch.no_grad()
    def generate(self, ids, n_new):
        """Greedy decoding: (tokens [B, n_new], logits [B, n_new - 1, vocab])."""
        toks = torch.empty(ids.shape[0], n_new, dtype=torch.long, device=ids.device)
        toks[:, 0] = self.prefill(ids)
        logits = []
        for j in range(1, n_new):
            logits.append(self.step(toks[:, j - 1]))
            toks[:, j] = self._next
        return toks, torch.stack(logits, 1)

    def close(self):
        """Releases the captured graph (its memory pool)."""
        self._graph = None

    def kv_bytes(self):
        return sum(c.nbytes() for c in self.caches())
