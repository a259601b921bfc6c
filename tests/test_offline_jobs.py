"""Accuracy job runner and result collectors (CPU, tiny random model)."""

import json

import pytest
import torch
from transformers import Qwen2Config, Qwen2ForCausalLM

from kvserve_hpdps_b200.offline import accuracy_jobs as AJ


@pytest.fixture(scope="module")
def model():
    cfg = Qwen2Config(vocab_size=256, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=32,
                      max_position_embeddings=2048)
    torch.manual_seed(0)
    return Qwen2ForCausalLM(cfg).eval()


def test_jobs_run_resume_and_collect(model, tmp_path):
    out = str(tmp_path / "acc.jsonl")
    jobs = AJ.expand_jobs(["default", "kivi", "custom"], ["synthetic"],
                          grid={"kivi": [{"nbits": 2}, {"nbits": 4}]})
    assert [(j.method, j.params.get("nbits")) for j in jobs] == \
        [("default", None), ("kivi", 2), ("kivi", 4), ("custom", None)]
    scores = torch.full((2, 2), 0.5)
    kw = dict(tokens=64, prompts=2, max_new_tokens=4)
    rows = AJ.run_jobs(model, "tiny", jobs, out, scores, **kw)
    assert len(rows) == 4 and len(AJ.read_rows(out)) == 4
    assert AJ.run_jobs(model, "tiny", jobs, out, scores, **kw) == []  # resumed: nothing left
    summary = AJ.collect(AJ.read_rows(out))
    assert [s["method"] for s in summary][0] == "default"
    d = summary[0]
    assert d["accuracy"] == 100.0 and d["accuracy_vs_default"] == 100.0  # exact cache
    for s in summary:
        assert s["backend"] == "prompt-set" and 0.0 <= s["accuracy"] <= 100.0
        assert s["compression_ratio"] >= 1.0
    kivi = [s for s in summary if s["method"] == "kivi"]
    assert {json.loads(s["config"])["nbits"] for s in kivi} == {2, 4}
    csv_path = tmp_path / "summary.csv"
    AJ.write_csv(summary, str(csv_path))
    assert csv_path.read_text().splitlines()[0].startswith("model,task,method,config")


def test_prompt_files_and_unknown_tasks(tmp_path):
    p = tmp_path / "p.jsonl"
    p.write_text('{"input_ids": [1, 2, 3]}\n{"input_ids": [4, 5]}\n')
    got = AJ.load_prompts(str(p), 256, count=0)
    assert [t.tolist() for t in got] == [[1, 2, 3], [4, 5]]
    q = tmp_path / "p.json"
    q.write_text("[[7, 8], [9]]")
    assert [t.tolist() for t in AJ.load_prompts(str(q), 256, count=1)] == [[7, 8]]
    with pytest.raises(ValueError, match="unknown task"):
        AJ.load_prompts("no_such_task", 256)


def test_collect_speed_reads_component_speed_lines():
    lines = ['noise', '{"stage": "quant", "ms": 0.4, "gbps": 1174.4, "layers": 28, '
             '"tokens": 8192, "heads": 4, "engine": 0}',
             '{"stage": "dequant", "ms": 0.25, "gbps": 1879.0, "layers": 28, "tokens": 8192, '
             '"heads": 4, "engine": 0}',
             '{"stage": "summary", "code_width": 8, "compression_ratio": 8.53}']
    rows = AJ.collect_speed(lines, source="run1")
    assert [r["stage"] for r in rows] == ["quant", "dequant"]
    assert rows[0]["compression_ratio"] == 8.53 and rows[1]["code_width"] == 8


def test_cli_collect(tmp_path, capsys):
    res = tmp_path / "r.jsonl"
    res.write_text("\n".join(json.dumps(r) for r in [
        {"key": "a", "model": "m", "task": "t", "method": "default", "config": {},
         "accuracy": 80.0, "backend": "lm-eval"},
        {"key": "b", "model": "m", "task": "t", "method": "custom", "config": {"x": 1},
         "accuracy": 60.0, "compression_ratio": 5.0, "backend": "lm-eval"}]) + "\n")
    assert AJ.main(["collect", str(res)]) == 0
    out = capsys.readouterr().out.splitlines()
    assert out[0].startswith("model,task,method") and ",75.0," in out[2]


def test_task_file_jobs_score_with_each_method(model, tmp_path):
    """A task file as a job's task: accuracy = the task's score x100."""
    from kvserve_hpdps_b200.offline.lm_harness import CacheMethodModel
    cm = CacheMethodModel(model, "default")
    docs = []
    for i in range(3):
        ctx = torch.randint(0, 256, (40,), generator=torch.Generator().manual_seed(i)).tolist()
        docs.append({"context_ids": ctx,
                     "answers_ids": [cm.generate(torch.tensor([ctx]), 4)[0].tolist()]})
    task = tmp_path / "qa.json"
    task.write_text(json.dumps({"kind": "generate", "max_new_tokens": 4, "docs": docs}))
    jobs = AJ.expand_jobs(["default", "custom"], [str(task)])
    rows = AJ.run_jobs(model, "tiny", jobs, str(tmp_path / "acc.jsonl"),
                       torch.full((2, 2), 0.5), limit=2)
    assert [r["backend"] for r in rows] == ["task-file", "task-file"]
    assert rows[0]["accuracy"] == 100.0 and rows[0]["docs"] == 2
    assert 0.0 <= rows[1]["accuracy"] <= 100.0 and rows[1]["compression_ratio"] > 1.0
