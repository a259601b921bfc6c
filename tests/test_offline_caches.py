"""Offline KV caches on a tiny random Hugging Face model (CPU): the
KVServe hybrid cache, KIVI, CacheGen, DuoAttention, the transforms, the
accuracy harness and the per-method CR tool."""

import pytest
import torch
from transformers import DynamicCache, Qwen2Config, Qwen2ForCausalLM

from kvserve_hpdps_b200.offline import caches as C
from kvserve_hpdps_b200.offline.lm_harness import evaluate_method, make_cache

L, H, D = 2, 2, 32


@pytest.fixture(scope="module")
def model():
    cfg = Qwen2Config(vocab_size=256, hidden_size=128, intermediate_size=256, num_hidden_layers=L,
                      num_attention_heads=4, num_key_value_heads=H, head_dim=D,
                      max_position_embeddings=2048)
    torch.manual_seed(0)
    return Qwen2ForCausalLM(cfg).eval()


def _kv(t=300, seed=1):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(1, H, t, D, generator=g)
    k[..., :2] *= 12  # outlier channels
    return k, torch.randn(1, H, t, D, generator=g)


def test_custom_cache_prefill_exact_then_reconstructs():
    scores = torch.tensor([[0.1, 0.9], [0.8, 0.2]])
    cfg = C.CustomCacheConfig("hadamard", scores, 0.5, 255, 255, 15, 15)
    cache = C.CustomCache(cfg)
    k, v = _kv()
    for layer in range(L):
        rk, rv = cache.update(k, v, layer)
        assert torch.equal(rk, k) and torch.equal(rv, v)  # prefill attends to exact KV
    pack = cache.packs[0]
    assert pack["low"].tolist() == [True, False]  # lowest-scored head of layer 0
    assert int(pack["k_low"][0].max()) <= 15 and int(pack["k_high"][0].max()) > 15
    nk, nv = _kv(1, seed=2)
    kk, vv = cache.update(nk, nv, 0)
    assert kk.shape[-2] == 301 and cache.get_seq_length(0) == 301
    assert torch.equal(kk[:, :, -1:], nk)
    err_hi = ((kk[:, 1, :300] - k[:, 1]) ** 2).mean() / (k[:, 1] ** 2).mean()
    err_lo = ((kk[:, 0, :300] - k[:, 0]) ** 2).mean() / (k[:, 0] ** 2).mean()
    assert float(err_hi) < 1e-3 < float(err_lo) < 0.05
    assert cache.compute_compression_ratio() > 1.5


def test_custom_config_checks():
    with pytest.raises(ValueError):
        C.CustomCacheConfig(transform_type="fft")
    with pytest.raises(ValueError):
        C.CustomCacheConfig(high_key_max_value=4, low_key_max_value=8)
    with pytest.raises(ValueError):
        C.CustomCacheConfig(axis_key=[4])


def test_transforms_invert():
    x = torch.randn(1, H, 10, D)
    had = C.HeadHadamard(0x3333)
    assert torch.allclose(had.inverse(had.transform(x, 3), 3), x, atol=1e-5)
    aff = C.AffineTransform(D, "diag", clip_init=100.0)
    aff.params[0] = {"log_scale": torch.linspace(-1, 1, D), "clip_k": torch.full((D,), 50.0),
                     "clip_v": torch.full((D,), 50.0)}
    assert torch.allclose(aff.inverse(aff.transform(x, 0, "k"), 0), x, atol=1e-5)
    full = C.AffineTransform(D, "full", learnable_clip=False)
    w = torch.eye(D) + 0.1 * torch.randn(D, D, generator=torch.Generator().manual_seed(0))
    full.params[1] = {"linear.weight": w}
    assert torch.allclose(full.inverse(full.transform(x, 1), 1), x, atol=1e-4)
    clipped = C.AffineTransform(D, "diag", clip_init=1.0).transform(x * 10, 5, "v")
    assert float(clipped.abs().max()) <= 1.0 + 1e-6


def test_kivi_residual_window():
    cache = C.KIVICache(C.KIVICacheConfig(nbits=2, q_group_size=32, residual_length=128))
    k, v = _kv(300)
    cache.update(k, v, 0)
    layer = cache.layers[0]
    assert layer.qk[0].shape[2] * layer.qk[0].shape[3] == 256 and layer.keys.shape[-2] == 44
    for i in range(84):  # the window reaches 128 tokens and folds into the codes
        nk, nv = _kv(1, seed=10 + i)
        kk, _ = cache.update(nk, nv, 0)
        assert kk.shape[-2] == 301 + i
    assert layer.keys.shape[-2] == 0
    assert layer.qk[0].shape[2] * layer.qk[0].shape[3] == 384
    assert 1.5 < cache.compute_compression_ratio() < 8.5


def test_cachegen_bins_and_codes():
    bins = C.cachegen_bins(C.CacheGenCacheConfig(model_layers=28, quantization_level=1))
    assert [b["k"] for b in bins].count(16) == int(28 * 0.63)
    assert [b["v"] for b in bins].count(16) == max(2, int(28 * 0.15))
    assert all(b == {"k": 32, "v": 32} for b in
               C.cachegen_bins(C.CacheGenCacheConfig(model_layers=4, quantization_level=3)))
    cache = C.CacheGenCache(C.CacheGenCacheConfig(model_layers=1, quantization_level=3))
    k, v = _kv(64)
    cache.update(k, v, 0)
    kk, vv = cache.update(*_kv(1, 3), 0)
    rel = ((kk[:, :, :64] - k) ** 2).sum() / (k ** 2).sum()
    assert float(rel) < 0.05 and cache.compute_compression_ratio() > 2


def test_search_hyperplane_separates():
    x = torch.randn(3, 50, 16) + 2.0
    y = C.search_hyperplane(x)
    assert bool((torch.bmm(x, y.unsqueeze(-1)) < 0).all())


def test_duoattention_drops_middle_tokens(model):
    scores = torch.tensor([[0.0, 1.0], [1.0, 0.0]])
    ids = torch.randint(0, 256, (1, 200), generator=torch.Generator().manual_seed(4))
    cache = C.DuoAttentionCache(C.DuoAttentionCacheConfig(scores, 0.5, sink_size=16,
                                                          recent_size=32))
    hooks = C.enable_query_capture(model)
    try:
        out = model(ids, past_key_values=cache, use_cache=True)
        keys_before = cache.layers[0].keys.clone()
        model(out.logits[:, -1:].argmax(-1), past_key_values=cache, use_cache=True)
    finally:
        for h in hooks:
            h.remove()
    keys = cache.layers[0].keys
    # streaming head 0 of layer 0: tokens 16..168 replaced by one fake key
    mid = keys[0, 0, 16:201 - 32]
    assert torch.equal(mid, mid[:1].expand_as(mid))
    assert torch.equal(keys[0, 1, :200], keys_before[0, 1])  # retrieval head untouched
    assert cache.compute_compression_ratio() > 1.0


def test_harness_default_is_exact_and_methods_run(model):
    prompts = [torch.randint(0, 256, (160,), generator=torch.Generator().manual_seed(s))
               for s in range(2)]
    base = evaluate_method(model, prompts, "default", max_new_tokens=4)
    assert base.accuracy == 100.0 and base.top1_agreement == 1.0 and abs(base.kl) < 1e-6
    scores = torch.rand(L, H, generator=torch.Generator().manual_seed(1))
    cr = evaluate_method(model, prompts, "custom", scores=scores, max_new_tokens=4,
                         transform_type="hadamard", heads_selection=0.5,
                         high_key_max_value=16, high_value_max_value=16,
                         low_key_max_value=8, low_value_max_value=8)
    assert cr.compression_ratio > 2 and 0 <= cr.accuracy <= 100
    assert isinstance(make_cache("default", L), DynamicCache)
    with pytest.raises(ValueError):
        make_cache("zip", L)


def test_cr_methods_tool_runs():
    from kvserve_hpdps_b200.offline import cr_methods
    m, spec = cr_methods.random_model("Llama-3-8B", layers=2, hidden=256)
    assert m.config.num_key_value_heads == spec.num_kv_heads == 8
    rows = cr_methods.run(m, [torch.randint(0, 1000, (300,))], torch.rand(2, 8),
                          methods=("custom", "kivi", "cachegen"), max_new_tokens=2)
    assert [r["method"] for r in rows] == ["custom", "kivi", "cachegen"]
    assert all(r["compression_ratio"] > 1.5 for r in rows)


def _duo_brute_force(model, ids, q_len):
    """The scorer's definition evaluated directly: stored layer inputs, the
    full repeated query matrix, every query row's attention computed."""
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb
    cfg = model.config
    n_q, n_kv = cfg.num_attention_heads, cfg.num_key_value_heads
    hs = model(ids.view(1, -1), output_hidden_states=True).hidden_states[:-1]
    out = torch.zeros(len(hs), n_kv)
    pos = torch.arange(q_len).view(1, -1)
    for i, h in enumerate(hs):
        layer = model.model.layers[i]
        h = layer.input_layernorm(h)
        q = layer.self_attn.q_proj(h).view(1, -1, n_q, D).mean(1, keepdim=True)
        k = layer.self_attn.k_proj(h).view(1, -1, n_kv, D).mean(1, keepdim=True)
        q = q.repeat(1, q_len, 1, 1).transpose(1, 2)
        k = k.repeat(1, q_len, 1, 1).transpose(1, 2)
        cos, sin = model.model.rotary_emb(h, pos)
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
        k = k.repeat_interleave(n_q // n_kv, dim=1)
        w = (q @ k.transpose(2, 3) / D ** 0.5).softmax(-1)[0, :, -1]  # last query row
        out[i] = w.cumsum(-1).mean(-1).view(n_kv, -1).mean(1)
    return out


def test_duo_scores_on_the_fly_match_definition(model, tmp_path, monkeypatch):
    from kvserve_hpdps_b200.compression.head_scores import DuoConfigGenerator
    from kvserve_hpdps_b200.offline.duo_scores import duo_scores_on_the_fly, main, \
        save_scores_csv
    g = torch.Generator().manual_seed(7)
    samples = [torch.randint(0, 256, (n,), generator=g) for n in (90, 140)]
    with torch.no_grad():
        want = sum(_duo_brute_force(model, s, 64) for s in samples) / 2
    got = duo_scores_on_the_fly(model, samples, q_len=64, max_tokens=512)
    assert got.shape == (L, H)
    assert torch.allclose(got, want, atol=1e-5, rtol=1e-5)
    assert bool(((got > 1 / 64 - 1e-6) & (got <= 1 + 1e-6)).all())
    # truncation to max_tokens, the class entry point and the CSV round trip
    short = duo_scores_on_the_fly(model, [samples[1][:50]], q_len=64)
    assert torch.allclose(DuoConfigGenerator.duo_attention_on_the_fly(
        model, [samples[1]], q_len=64, max_tokens=50), short)
    monkeypatch.chdir(tmp_path)
    save_scores_csv(got, "tiny-duo-model_scores.csv")
    back = DuoConfigGenerator.get_scores_from_csv("/models/tiny-duo-model")
    assert torch.allclose(back, got)
    assert main(["--model", "random:Qwen2.5-7B", "--layers", "2", "--hidden", "512",
                 "--q-len", "32", "--max-tokens", "64", "--random-samples", "1",
                 "--out", "r.csv"]) == 0
    assert (tmp_path / "r.csv").read_text().count("\n") == 2


def test_component_speed_methods_run_on_cpu(capsys):
    import json

    from kvserve_hpdps_b200.offline import component_speed as CS
    rows = CS.run_methods(layers=2, tokens=256, heads=2, iters=1, warmup=1, device="cpu")
    got = {(r["method"], r["phase"]) for r in rows}
    assert got == {(m, p) for m in CS.METHODS for p in ("compress", "reconstruct")}
    assert all(r["ms"] > 0 and r["gbps"] > 0 for r in rows)
    crs = {r["method"]: r["compression_ratio"] for r in rows if r.get("compression_ratio")}
    assert set(crs) == {"custom", "kivi", "cachegen"} and min(crs.values()) > 1.5
    with pytest.raises(ValueError):
        CS.run_methods(("zip",), layers=1, tokens=16, heads=1, device="cpu")
    assert CS.main(["--methods", "minmax", "--layers", "1", "--tokens", "64", "--heads", "1",
                    "--iters", "1", "--warmup", "1", "--device", "cpu"]) == 0
    assert [json.loads(x)["phase"] for x in capsys.readouterr().out.splitlines()] == \
        ["compress", "reconstruct"]


def test_lm_eval_model_args_split():
    """lm-eval model_args as the reference's wrapper takes them (bare) or
    prefixed: cache parameters go to the method's config, the rest to HFLM."""
    from kvserve_hpdps_b200.offline.lm_harness import split_cache_args
    p, scores, rest = split_cache_args("custom", {
        "pretrained": "m", "transform_type": "hadamard", "cache_heads_selection": 0.3,
        "high_key_max_value": 16, "scores": "Qwen2.5-7B-Instruct", "dtype": "bfloat16"})
    assert p == {"transform_type": "hadamard", "heads_selection": 0.3, "high_key_max_value": 16}
    assert scores == "Qwen2.5-7B-Instruct" and rest == {"pretrained": "m", "dtype": "bfloat16"}
    p, _, rest = split_cache_args("kivi", {"nbits": 2, "q_group_size": 32, "batch_size": 4})
    assert p == {"nbits": 2, "q_group_size": 32} and rest == {"batch_size": 4}
    p, _, rest = split_cache_args("default", {"nbits": 2})
    assert p == {} and rest == {"nbits": 2}
    with pytest.raises(ValueError):
        split_cache_args("zip", {})


def test_register_lm_eval_model_runs_with_a_cache(model, monkeypatch):
    """``register_lm_eval`` against a stand-in of lm-eval's registry and HFLM
    base class (lm-eval itself is not installed): the registered class takes
    the reference wrapper's bare model_args, builds the cache method, and its
    ``_model_generate`` (what lm-eval calls for generation tasks) decodes with
    that cache -- greedy tokens identical to the plain model for the default
    cache, and mostly identical for the hybrid cache."""
    import sys
    import types

    registry: dict = {}

    def register_model(name):
        def deco(cls):
            registry[name] = cls
            return cls
        return deco

    class HFLM:  # what the registered class needs from lm-eval's base class
        def __init__(self, pretrained=None, batch_size=1, **kw):
            self.model = pretrained
            self.batch_size = batch_size
            self.tokenizer = types.SimpleNamespace(pad_token_id=0)

    mods = {"lm_eval": types.ModuleType("lm_eval"),
            "lm_eval.api": types.ModuleType("lm_eval.api"),
            "lm_eval.api.registry": types.ModuleType("lm_eval.api.registry"),
            "lm_eval.models": types.ModuleType("lm_eval.models"),
            "lm_eval.models.huggingface": types.ModuleType("lm_eval.models.huggingface")}
    mods["lm_eval.api.registry"].register_model = register_model
    mods["lm_eval.models.huggingface"].HFLM = HFLM
    for k, v in mods.items():
        monkeypatch.setitem(sys.modules, k, v)
    from kvserve_hpdps_b200.offline.lm_harness import register_lm_eval
    cls = register_lm_eval()
    assert registry["my_custom_model"] is cls
    ctx = torch.randint(0, 256, (1, 200), generator=torch.Generator().manual_seed(3))
    plain = model.generate(input_ids=ctx, max_length=224, do_sample=False, pad_token_id=0)
    lm = cls(pretrained=model, batch_size=1, cache_type="default")
    out = lm._model_generate(ctx, 224, None)
    assert torch.equal(out, plain)
    lm = cls(pretrained=model, batch_size=1, cache_type="custom", transform_type="hadamard",
             heads_selection=0.5, high_key_max_value=255, high_value_max_value=255,
             low_key_max_value=15, low_value_max_value=15,
             scores=None)
    out = lm._model_generate(ctx, 224, None)
    assert out.shape == plain.shape
    assert torch.equal(out[:, :200], ctx)
    agree = float((out[:, 200:] == plain[:, 200:]).float().mean())
    assert agree > 0.5, agree
    assert lm._kvs.last_cache is not None and type(lm._kvs.last_cache).__name__ == "CustomCache"
