"""Local task accuracy, the model-based evaluators and the model search
(CPU, tiny random-init model)."""

import json
import random

import pytest
import torch
from transformers import Qwen2Config, Qwen2ForCausalLM

from kvserve_hpdps_b200.offline import param_search as PS
from kvserve_hpdps_b200.offline import tasks as T
from kvserve_hpdps_b200.offline.lm_harness import CacheMethodModel

HIGH = {"transform_type": "hadamard", "heads_selection": 0.0, "high_key_max_value": 255,
        "high_value_max_value": 255, "low_key_max_value": 255, "low_value_max_value": 255,
        "axis_key": [2], "axis_value": [1, 3]}
LOW = {"transform_type": "none", "heads_selection": 1.0, "high_key_max_value": 2,
       "high_value_max_value": 2, "low_key_max_value": 2, "low_value_max_value": 2,
       "axis_key": [2], "axis_value": [1, 3]}


@pytest.fixture(scope="module")
def model():
    cfg = Qwen2Config(vocab_size=128, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=32,
                      max_position_embeddings=1024)
    torch.manual_seed(0)
    return Qwen2ForCausalLM(cfg).eval()


def _ctx(i, n=48):
    g = torch.Generator().manual_seed(100 + i)
    return torch.randint(0, 128, (n,), generator=g).tolist()


def _gen_task(model, path, n_docs=6, new=6):
    """Answers are the default cache's own greedy continuations."""
    cm = CacheMethodModel(model, "default")
    docs = []
    for i in range(n_docs):
        ctx = _ctx(i)
        out = cm.generate(torch.tensor([ctx]), new)[0].tolist()
        docs.append({"context_ids": ctx, "answers_ids": [out]})
    path.write_text(json.dumps({"name": "gen", "kind": "generate", "max_new_tokens": new,
                                "docs": docs}))
    return str(path)


def _choice_task(model, path, n_docs=5):
    """Gold = the continuation the default cache likes best."""
    runner = T.TaskRunner(CacheMethodModel(model, "default"))
    lines = []
    for i in range(n_docs):
        ctx = _ctx(10 + i, 40)
        choices = [_ctx(50 + 3 * i + j, 3) for j in range(3)]
        lls = [runner.continuation_logprob(torch.tensor([ctx]), c) for c in choices]
        lines.append(json.dumps({"context_ids": ctx, "choices_ids": choices,
                                 "gold": max(range(3), key=lambda j: lls[j])}))
    path.write_text("\n".join(lines) + "\n")
    return str(path)


def test_answer_metrics():
    assert T.normalize_answer("The  Eiffel-Tower, in Paris!") == "eiffeltower in paris"
    assert T.token_f1("a b c".split(), "b c d".split()) == pytest.approx(2 / 3)
    assert T.token_f1([], [1]) == 0.0
    s = T.text_scores("It is the Eiffel Tower.", ["Eiffel Tower", "Louvre"])
    assert s["contains"] == 1.0 and s["exact_match"] == 0.0
    assert s["qa_f1"] == pytest.approx(2 * (2 / 4) * 1.0 / (2 / 4 + 1.0))
    assert T.text_scores("eiffel tower", ["The Eiffel Tower"])["exact_match"] == 1.0
    ids = T.id_scores([5, 6, 7, 8], [[6, 7], [5, 6]])
    assert ids == {"qa_f1": pytest.approx(2 / 3), "exact_match": 1.0, "contains": 1.0}
    assert T._cut_at_stop([1, 2, 3, 4, 2, 3], [[2, 3]]) == [1]


def test_stratified_sample_is_the_seeded_interval_draw():
    """Same indices as seeding Python's generator once and drawing one index
    per interval, task after task (the reference's procedure)."""
    rng = random.Random(42)
    a = PS.stratified_indices(103, 10, rng)
    b = PS.stratified_indices(37, 5, rng)
    random.seed(42)
    want = []
    for n, k in ((103, 10), (37, 5)):
        step = n / k
        want.append([random.randrange(int(i * step), min(max(int((i + 1) * step),
                                                              int(i * step) + 1), n))
                     for i in range(k)])
    assert [a, b] == want
    for i, x in enumerate(a):
        assert int(i * 10.3) <= x < int((i + 1) * 10.3)
    assert PS.stratified_indices(4, 10, random.Random(0)) == [0, 1, 2, 3]


def test_task_files_load_and_are_told_from_prompt_sets(tmp_path):
    g = tmp_path / "g.jsonl"
    g.write_text('{"context": "q?", "answers": ["a"]}\n{"context": "r?", "answers": ["b"]}\n')
    t = T.load_task(str(g), max_new_tokens=4)
    assert (t.name, t.kind, t.metric, t.max_new_tokens, len(t.docs)) == ("g", "generate",
                                                                          "qa_f1", 4, 2)
    c = tmp_path / "c.json"
    c.write_text(json.dumps([{"context_ids": [1], "choices_ids": [[2], [3]], "gold": 0}]))
    assert T.load_task(str(c)).kind == "choice" and T.load_task(str(c)).metric == "acc"
    p = tmp_path / "p.jsonl"
    p.write_text('{"input_ids": [1, 2]}\n')
    assert T.is_task_file(str(g)) and T.is_task_file(str(c))
    assert not T.is_task_file(str(p)) and not T.is_task_file(str(tmp_path / "none.json"))
    with pytest.raises(ValueError, match="kind"):
        T.LocalTask("x", "rank", [{}])
    with pytest.raises(ValueError, match="tokenizer"):
        T.TaskRunner(CacheMethodModel.__new__(CacheMethodModel)).score_doc(t, t.docs[0])


def test_runner_scores_default_cache_exactly(model, tmp_path):
    gen = T.load_task(_gen_task(model, tmp_path / "gen.json"))
    ch = T.load_task(_choice_task(model, tmp_path / "ch.jsonl"))
    runner = T.TaskRunner(CacheMethodModel(model, "default"))
    r = runner.run(gen)
    assert r["score"] == 1.0 and r["exact_match"] == 1.0 and r["docs"] == 6
    assert runner.run(ch, [0, 2, 4]) == {"acc": 1.0, "score": 1.0, "docs": 3}
    # the continuation is scored through the method's cache after the prefill
    ctx = torch.tensor([_ctx(3, 40)])
    with torch.no_grad():
        full = model(torch.cat([ctx, torch.tensor([[7, 8, 9]])], 1)).logits[0].float()
    lp = torch.log_softmax(full, -1)
    want = float(lp[39, 7] + lp[40, 8] + lp[41, 9])
    assert runner.continuation_logprob(ctx, [7, 8, 9]) == pytest.approx(want, abs=1e-3)


def test_accuracy_evaluator_normalises_against_the_default_cache(model, tmp_path):
    _gen_task(model, tmp_path / "gen.json")
    _choice_task(model, tmp_path / "ch.jsonl")
    ev = PS.AccuracyEvaluator("Qwen2.5-7B-Instruct", ["gen", "ch"], limit=4, random_seed=42,
                              model=model, task_dirs=[str(tmp_path)])
    assert set(ev.samples) == {"gen", "ch"} and len(ev.samples["gen"]) == 4
    assert ev.default_scores == [1.0, 1.0]
    assert tuple(ev.scores.shape) == (2, 2)  # the package table cut to the model
    hi = ev.evaluate(HIGH)
    lo = ev.evaluate(LOW)
    assert 0.0 <= lo < hi <= 100.0 and hi >= 90.0
    with pytest.raises(ValueError, match="search parameters"):
        ev.evaluate({"heads_selection": 0.5})
    with pytest.raises(RuntimeError, match="lm-eval is not installed"):
        PS.AccuracyEvaluator("tiny", ["longbench_hotpotqa"], model=model)


def test_compression_evaluator_orders_precisions(model, tmp_path):
    path = _gen_task(model, tmp_path / "gen.json")
    ev = PS.CompressionEvaluator("Qwen2.5-7B-Instruct", path, model=model)
    assert ev.input_ids.shape == (1, 48)
    hi, lo = ev.evaluate(HIGH), ev.evaluate(LOW)
    assert 1.0 < hi < lo
    syn = PS.CompressionEvaluator("tiny", None, model=model, synthetic_tokens=96)
    assert syn.input_ids.shape == (1, 96) and syn.evaluate(HIGH) > 1.0


def test_model_search_writes_results_and_library(model, tmp_path):
    from kvserve_hpdps_b200.offline.search import run_model_search
    _gen_task(model, tmp_path / "gen.json", n_docs=3, new=4)
    space = {"hybrid_ratio": [0.0, 1.0], "high_key_max_value": [16], "high_value_max_value": [16],
             "low_key_max_value": [4], "low_value_max_value": [4]}
    out = tmp_path / "out"
    res = run_model_search("Qwen2.5-7B-Instruct", ["gen"], 3.0, str(out), budget=2,
                           space=space, limit=3, task_dirs=(str(tmp_path),), model=model)
    assert res["tasks"] == ["gen"] and res["default_scores"] == [1.0]
    assert res["evaluations"] == 2
    saved = json.loads((out / "tolerance_3_results.json").read_text())
    assert saved["threshold"] == 97.0 and len(saved["history"]) == 2
    lib = json.loads((out / "profile_library.json").read_text())
    assert lib and (out / "cr_cache.csv").exists()
    # the controller compares fractions (accuracy_requirement 0.92): task
    # accuracy x100 of the default cache goes into the library as a fraction
    accs = [p["quality_metrics"]["accuracy"] for b in lib["accuracy_buckets"]
            for p in b["pareto_profiles"]]
    assert accs and all(0.0 <= a <= 1.0 for a in accs)
    for h in saved["history"]:
        assert h["compression_ratio"] > 1.0 and 0.0 <= h["accuracy"] <= 100.0


def test_text_tasks_through_a_tokenizer(model, tmp_path):
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast
    words = ["<unk>", "where", "is", "the", "tower", "paris", "rome", "?"] + \
        [f"w{i}" for i in range(120)]
    tk = Tokenizer(models.WordLevel({w: i for i, w in enumerate(words)}, unk_token="<unk>"))
    tk.pre_tokenizer = pre_tokenizers.Whitespace()
    tok = PreTrainedTokenizerFast(tokenizer_object=tk, unk_token="<unk>")
    cm = CacheMethodModel(model, "default")
    ctx = "where is the tower ? " + " ".join(f"w{i}" for i in range(30))
    ids = tok(ctx)["input_ids"]
    out = tok.decode(cm.generate(torch.tensor([ids]), 3)[0].tolist(), skip_special_tokens=True)
    docs = [{"context": ctx, "answers": [out]},
            {"context": ctx, "choices": ["paris", "rome"], "gold": 0}]
    (tmp_path / "t.json").write_text(json.dumps({"kind": "generate", "max_new_tokens": 3,
                                                 "docs": docs[:1]}))
    runner = T.TaskRunner(cm, tok)
    assert runner.run(T.load_task(str(tmp_path / "t.json")))["score"] == 1.0
    (tmp_path / "c.json").write_text(json.dumps({"kind": "choice", "docs": docs[1:]}))
    r = runner.run(T.load_task(str(tmp_path / "c.json")))
    assert r["acc"] in (0.0, 1.0)
