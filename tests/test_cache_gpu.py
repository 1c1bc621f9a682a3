"""CompressedKV on the B200 kernels: prefill, append across page boundaries and
raw-pool growth stay exact (reference tests/test_exactkv.py:81-104)."""
import numpy as np
import pytest
import torch

import exactkv_b200 as ekv
from exactkv_b200 import kernels
from gpu_util import same_bits, to_bits
from oracle import codec as ocodec

pytestmark = pytest.mark.gpu


def test_cache_append_and_pool_growth():
    """Many rows that do not fit and a tiny initial pool: the pool must grow and
    decode and attention must stay exact."""
    g = torch.Generator().manual_seed(2)
    B, H, D, T0, TS = 2, 4, 128, 1000, 1200

    def make(n):
        x = torch.randn(B, n, H, D, generator=g).to(torch.bfloat16)
        x[torch.rand(B, n, H, generator=g) < 0.1, 7] = 1e-30     # forces raw rows
        return x.cuda()

    c, r = ekv.CompressedKV(B, TS, H, D, reserve=0.001), ekv.BF16KV(B, TS, H, D)
    x0 = make(T0)
    for b in range(B):
        c.prefill_slot(b, x0[b:b + 1].contiguous())
        r.prefill_slot(b, x0[b:b + 1].contiguous())
    xs = make(TS - T0)
    q = torch.randn(B, 32, D, generator=g).to(torch.bfloat16).cuda()
    for t in range(TS - T0):
        c.append(xs[:, t].contiguous())
        r.append(xs[:, t].contiguous())
        ekv.check_overflow([c])
        if t % 37 == 0 or t == TS - T0 - 1:
            assert same_bits(kernels.decode_to_bf16(c.buffers(), c.T), r.buf[:, :c.T]), t
            assert same_bits(ekv.decode_attention(q, c, c), ekv.decode_attention(q, r, r)), t
    assert c.grows > 0
    kernels.check_status()


def test_prefill_equals_encode_reference_bytes():
    """Slot-by-slot prefill writes the bytes encode_reference gives for the whole
    batch, rowoff and raw included (slots follow (sequence, page, head) order)."""
    g = torch.Generator().manual_seed(3)
    B, T, H = 3, 512, 4
    x = torch.randn(B, T, H, 128, generator=g).to(torch.bfloat16)
    x[torch.rand(B, T, H, generator=g) < 0.05, 11] = 1e-30
    ref = ocodec.encode(to_bits(x))
    x = x.cuda()
    c = ekv.CompressedKV(B, T, H, 128, reserve=0.2)
    for b in range(B):
        c.prefill_slot(b, x[b:b + 1].contiguous())
    for f in ("sm", "code", "base", "rowmask", "rowoff"):
        assert np.array_equal(getattr(c, f).cpu().numpy(), ref[f]), f
    n = int(c.cnt.item())
    assert n == ref["raw"].shape[0]
    assert np.array_equal(to_bits(c.raw[:n]), ref["raw"])
    kernels.check_status()


def test_bits_per_value_and_nbytes():
    c = ekv.CompressedKV(2, 256, 2, 128)
    assert c.nbytes() == 2 * 256 * 2 * (128 + 64) + 2 * 16 * 2 * (128 + 8) + c.raw.numel() * 2
    x = torch.randn(1, 64, 2, 128).to(torch.bfloat16).cuda()
    enc = ekv.encode_reference(x)
    assert 12.5 <= ekv.bits_per_value(enc) < 13.5


def test_prefill_from_hf_layout_view():
    """Prefill straight from a model's [1, H, T, D] cache through a transposed view
    (the encoder reads it by strides) writes the same bytes as from a contiguous
    [1, T, H, D] copy."""
    from exactkv_b200 import synthetic
    T, H = 1000, 4
    x = synthetic.make_kv(2, T, H, seed=81, key=True)                 # [B, T, H, D]
    hf = x.transpose(1, 2).contiguous()                               # [B, H, T, D], as HF stores it
    a = ekv.CompressedKV(2, 1024, H, 128)
    b = ekv.CompressedKV(2, 1024, H, 128)
    for s in range(2):
        a.prefill_slot(s, x[s:s + 1].contiguous())
        b.prefill_slot(s, hf[s:s + 1].transpose(1, 2))
    for f in ("sm", "code", "base", "rowmask", "rowoff", "raw", "cnt"):
        assert torch.equal(getattr(a, f), getattr(b, f)), f
