"""Engine (the reference's exactkv/engine.py interface) on tiny random-init models.

GPU: the compressed and the bf16 cache give the same greedy tokens and
bit-identical logits (reference tests/test_exactkv.py:107-122, which needs a
downloaded checkpoint; random init stands in for it here), for a Llama-3 and a
Qwen3 (q/k norm) layout, through the CUDA-graphed decode step; the graphed step
gives the same bits as the same step run eagerly, across raw-pool growth
(captured again) and page boundaries; the hooked (host-length) path runs too.
CPU: the constructor's model checks.
"""
import pytest
import torch

D = 128


def _tiny(kind, layers=2, hq=2, hkv=1, vocab=512, seed=0):
    from transformers import LlamaConfig, LlamaForCausalLM, Qwen3Config, Qwen3ForCausalLM
    common = dict(vocab_size=vocab, hidden_size=hq * D, intermediate_size=512, num_hidden_layers=layers,
                  num_attention_heads=hq, num_key_value_heads=hkv, head_dim=D, max_position_embeddings=4096,
                  rope_theta=5e5)
    torch.manual_seed(seed)
    if kind == "llama":
        return LlamaForCausalLM(LlamaConfig(**common))
    return Qwen3ForCausalLM(Qwen3Config(**common))


def test_engine_rejects_unsupported_models():
    from transformers import GPT2Config, GPT2LMHeadModel
    from exactkv_b200.engine import Engine
    with pytest.raises(ValueError):
        Engine(GPT2LMHeadModel(GPT2Config(n_layer=1, n_embd=64, n_head=2)), 1, 32)
    m = _tiny("llama")
    m.config.head_dim = 64
    with pytest.raises(ValueError):
        Engine(m, 1, 32)


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["llama", "qwen3"])
def test_engine_compressed_equals_bf16(kind):
    import exactkv_b200 as ekv
    model = _tiny(kind).to(device="cuda", dtype=torch.bfloat16).eval()
    g = torch.Generator(device="cuda").manual_seed(1)
    ids = torch.randint(10, 500, (3, 500), generator=g, device="cuda")
    out = {}
    for be in ("bf16", "exactkv"):
        eng = ekv.Engine(model, 3, 500 + 40, backend=be)
        out[be] = eng.generate(ids, 40)
        if be == "exactkv":
            assert eng.T == 539 and eng.kv_bytes() > 0
        del eng
    assert torch.equal(out["bf16"][0], out["exactkv"][0])
    assert torch.equal(out["bf16"][1].view(torch.int16), out["exactkv"][1].view(torch.int16))
    ekv.kernels.check_status()


@pytest.mark.gpu
def test_graphed_step_equals_eager_step_across_pool_growth():
    import exactkv_b200 as ekv
    model = _tiny("llama", layers=2).to(device="cuda", dtype=torch.bfloat16).eval()
    g = torch.Generator(device="cuda").manual_seed(4)
    ids = torch.randint(10, 500, (2, 300), generator=g, device="cuda")
    out = {}
    for graphs in (True, False):
        eng = ekv.Engine(model, 2, 300 + 80, graphs=graphs, check_pages=1)
        tok = eng.prefill(ids)
        logits = []
        for i in range(70):
            if i == 35:
                # a wider window: the next check must grow every pool after the graph
                # was captured, and the step is captured again
                eng.check_pages = 40
            logits.append(eng.step(tok))
            tok = logits[-1].argmax(-1)
        out[graphs] = torch.stack(logits, 1)
        assert eng.grows > 0 and eng.T == 370
        if graphs:
            assert eng.captures >= 2
        eng.close()
        del eng
    assert torch.equal(out[True].view(torch.int16), out[False].view(torch.int16))
    ekv.kernels.check_status()


@pytest.mark.gpu
def test_hooked_engine_runs_on_host_lengths():
    import exactkv_b200 as ekv
    model = _tiny("llama", layers=1).to(device="cuda", dtype=torch.bfloat16).eval()
    ids = torch.randint(10, 500, (2, 100), device="cuda")
    seen = []
    eng = ekv.Engine(model, 2, 140, before_step=lambda e, T: seen.append(T))
    toks, logits = eng.generate(ids, 20)
    assert seen == list(range(101, 120)) and eng.T == 119 and eng.captures == 0
    ref = ekv.Engine(model, 2, 140, backend="bf16", attn=ekv.decode_attention)
    toks2, logits2 = ref.generate(ids, 20)
    assert torch.equal(toks, toks2) and torch.equal(logits.view(torch.int16), logits2.view(torch.int16))
