"""Prefill/decode disaggregated serving on one box: TTFT with the
compressed KV connector.

Two vLLM V1 engines run as two processes on two GPUs: the producer
(``kv_producer``, prefill) and the consumer (``kv_consumer``, decode), each
with the connector loaded through ``kv_connector_module_path``.  Every
request is dispatched to both engines at the same moment with the same
``transfer_id``; the consumer's scheduler claims the prompt's KV as external
tokens and its worker waits for the producer's message, injects the KV and
computes the first output token.  TTFT of a request = time from dispatch
until the consumer returned its first token.

Model: the Qwen2.5-7B architecture with random-init weights
(``load_format="dummy"``, no checkpoint needed), synthetic prompts of uniform
token ids.  ``--impl reference`` loads the reference connector
(``kvserve_v1``) from ``baseline/_ref`` instead of this package's.

Example::

  python examples/pd_ttft.py --requests 32 --prompt-len 8192 --compression default
  python examples/pd_ttft.py --compression none          # raw KV over the NVLink ring
  python examples/pd_ttft.py --impl reference --compression none
  python examples/pd_ttft.py --tp 2 --gpus 0,1,2,3      # TP2 producer and consumer
  # across two nodes (consumer first), transport nccl:
  python examples/pd_ttft.py --role consumer --gpus 0 --kv-ip <consumer host> --transport nccl
  python examples/pd_ttft.py --role producer --gpus 0 --kv-ip <consumer host> --transport nccl

Prints one JSON line with p50 / p90 / mean TTFT, the producer-side prefill
latency, the agreement of the consumer's first token with the producer's own
greedy token (a full prefill without transfer; 1.0 is required for raw KV)
and an md5 fingerprint of the consumer's greedy outputs.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import multiprocessing as mp
import os
import statistics
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

QWEN25_7B = {
    "architectures": ["Qwen2ForCausalLM"], "model_type": "qwen2", "hidden_act": "silu",
    "hidden_size": 3584, "intermediate_size": 18944, "num_hidden_layers": 28,
    "num_attention_heads": 28, "num_key_value_heads": 4, "vocab_size": 152064,
    "max_position_embeddings": 32768, "rope_theta": 1000000.0, "rms_norm_eps": 1e-6,
    "tie_word_embeddings": False, "torch_dtype": "bfloat16", "use_sliding_window": False,
    "sliding_window": None, "max_window_layers": 28, "bos_token_id": 151643,
    "eos_token_id": 151645, "attention_dropout": 0.0, "initializer_range": 0.02,
    "use_cache": True,
}


LLAMA3_8B = {
    "architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_act": "silu",
    "hidden_size": 4096, "intermediate_size": 14336, "num_hidden_layers": 32,
    "num_attention_heads": 32, "num_key_value_heads": 8, "vocab_size": 128256,
    "max_position_embeddings": 32768, "rope_theta": 500000.0, "rms_norm_eps": 1e-5,
    "tie_word_embeddings": False, "torch_dtype": "bfloat16", "bos_token_id": 128000,
    "eos_token_id": 128009, "attention_dropout": 0.0, "initializer_range": 0.02,
    "use_cache": True, "head_dim": 128,
}

QWEN25_32B = dict(QWEN25_7B, hidden_size=5120, intermediate_size=27648, num_hidden_layers=64,
                  num_attention_heads=40, num_key_value_heads=8, max_window_layers=64)

ARCHS = {"qwen2.5-7b": ("Qwen2.5-7B-Instruct", QWEN25_7B),
         "llama-3-8b": ("Llama-3-8B-Instruct", LLAMA3_8B),
         "qwen2.5-32b": ("Qwen2.5-32B-Instruct", QWEN25_32B)}


def write_model_dir(path: str, config: dict = QWEN25_7B) -> str:
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(config, f)
    return path


def write_controller_library(path: str, model_name: str) -> str:
    """A profile library over hybrid_ratio 0 / 0.3 / 1.0 of the default
    quantizer (fused path, rANS), with the compression ratios measured by the
    handoff sweep on Qwen2.5-7B shapes and accuracy standing in as the
    reconstruction cosine; harmonic speed in MB/s of original KV."""
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    from kvserve_hpdps_b200.offline.library_export import build_library, write_library

    def spec(cfg):
        return {"enabled": True, "pipeline": ["quantizer", "codec"],
                "quantizer_config": dict(cfg, model_name=model_name),
                "codec_config": {"codec_type": "rans"}, "min_compress_size": 0}
    base = {"high_key_max_value": 12, "high_value_max_value": 8, "low_key_max_value": 6,
            "low_value_max_value": 4}
    evals = [{"candidate": f"h{hr}", "config": dict(base, hybrid_ratio=hr), "accuracy": acc,
              "compression_ratio": cr, "harmonic_speed_mbps": 4.0e5}
             for hr, acc, cr in ((0.0, 0.96, 6.4), (0.3, 0.95, 7.1), (1.0, 0.93, 11.0))]
    write_library(path, build_library(evals, model_name, spec_builder=spec))
    return path


def compression_spec(name: str, args=None):
    if name == "none":
        return None
    if name == "default":
        return "default"
    if name == "controller":  # slo 200 ms, accuracy 0.92
        return {"mode": "controller", "library_path": args.library, "epsilon": 0.1,
                "service_config": {"bandwidth_mbps": 10000, "slo_ms": 200.0,
                                   "accuracy_requirement": 0.92, "t_model_ms": 0.0}}
    if name == "quantizer":  # the reference's degraded custom pipeline (no codec)
        return {"enabled": True, "pipeline": ["quantizer"],
                "quantizer_config": {"hybrid_ratio": 0.8, "high_key_max_value": 12,
                                     "high_value_max_value": 8, "low_key_max_value": 6,
                                     "low_value_max_value": 4, "axis_key": "channel",
                                     "axis_value": "token", "split_type": "head"},
                "min_compress_size": 0}
    raise ValueError(name)


def engine(role: str, gpus: str, args, q_in, q_out) -> None:
    os.environ["CUDA_VISIBLE_DEVICES"] = gpus
    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    if args.impl == "reference":
        sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
        os.environ["PYTHONPATH"] = os.path.join(ROOT, "baseline", "_ref") + os.pathsep + \
            os.environ.get("PYTHONPATH", "")
    else:
        sys.path.insert(0, ROOT)
    try:
        from vllm import LLM, SamplingParams
        from vllm.sampling_params import RequestOutputKind
        from vllm.config import KVTransferConfig
        module = ("kvserve_v1.connector.compressed_kv_connector" if args.impl == "reference"
                  else "kvserve_hpdps_b200.connector.compressed_kv_connector")
        extra = {"compression": compression_spec(args.compression, args)}
        if args.impl != "reference":
            extra["transport"] = args.transport
        ktc = KVTransferConfig(kv_connector="CompressedKVConnector",
                               kv_connector_module_path=module,
                               kv_role="kv_producer" if role == "p" else "kv_consumer",
                               kv_rank=0 if role == "p" else 1, kv_parallel_size=2,
                               kv_ip=args.kv_ip, kv_port=args.port,
                               kv_connector_extra_config=extra,
                               kv_load_failure_policy=args.load_failure_policy)
        llm = LLM(model=args.model_dir, dtype="bfloat16", load_format="dummy",
                  skip_tokenizer_init=True,
                  max_model_len=max(args.prompt_len, args.prompt_len_max) + args.max_tokens + 64,
                  max_num_batched_tokens=max(args.prompt_len, args.prompt_len_max) + 64,
                  max_num_seqs=8,
                  gpu_memory_utilization=args.mem_util, enforce_eager=True,
                  enable_prefix_caching=False, kv_transfer_config=ktc, seed=0,
                  tensor_parallel_size=args.tp)
        q_out.put(("ready", role))
        eng = llm.llm_engine
        while True:
            msg = q_in.get()
            if msg[0] == "stop":
                break
            _, i, ids = msg
            sp = SamplingParams(max_tokens=1 if role == "p" else args.max_tokens, temperature=0.0,
                                detokenize=False, output_kind=RequestOutputKind.CUMULATIVE,
                                extra_args={"kv_transfer_params": {"transfer_id": f"req-{i}"}})
            # drive the engine step by step (one request in flight): the first
            # token's arrival is the TTFT even when more tokens follow
            eng.add_request(f"{role}{i}", {"prompt_token_ids": ids}, sp)
            t_first, toks = None, []
            while eng.has_unfinished_requests():
                for o in eng.step():
                    if o.outputs and len(o.outputs[0].token_ids) > len(toks):
                        toks = list(o.outputs[0].token_ids)  # cumulative outputs
                        if t_first is None:
                            t_first = time.time()
            q_out.put(("done", role, i, t_first or time.time(), toks, time.time()))
    except Exception:  # noqa: BLE001
        import traceback
        q_out.put(("error", role, traceback.format_exc()))


def _stats_summary():
    """With KVSERVE_*_STATS_PATH set (the engines inherit it), the summary of
    the stats rows they wrote: mean compression ratio and the median
    compress + comm + decompress path."""
    paths = [os.environ.get(f"KVSERVE_{k}_STATS_PATH") for k in ("COMPRESSION", "DECODE",
                                                                    "TRANSFER")]
    if not any(paths):
        return None
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    from kvserve_hpdps_b200.utils.stats import summarize
    return summarize(*paths)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--compression", choices=["default", "none", "quantizer", "controller"],
                    default="default")
    ap.add_argument("--arch", choices=sorted(ARCHS), default="qwen2.5-7b",
                    help="random-init architecture (Qwen2.5-7B, Llama-3-8B, Qwen2.5-32B)")
    ap.add_argument("--transport", default="auto", help="ours: auto | p2p | nccl")
    ap.add_argument("--requests", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--prompt-len", type=int, default=8192)
    ap.add_argument("--prompt-len-max", type=int, default=0,
                    help="lengths uniform in [--prompt-len, this] (config 3: 2048..16384)")
    ap.add_argument("--max-tokens", type=int, default=1)
    ap.add_argument("--gpus", default="0,1",
                    help="producer GPUs then consumer GPUs (tp of each; one role: its tp GPUs)")
    ap.add_argument("--tp", type=int, default=1, help="tensor-parallel size of each engine")
    ap.add_argument("--load-failure-policy", default="fail", choices=["fail", "recompute"],
                    help="decode engine's answer to KV that did not arrive intact (fail: the "
                         "request ends with an error, so a measured run shows every failure)")
    ap.add_argument("--role", choices=["both", "producer", "consumer"], default="both",
                    help="producer / consumer: run one engine here and pair with --kv-ip "
                         "(the consumer's host) across nodes")
    ap.add_argument("--kv-ip", default="127.0.0.1", help="the consumer engine's host")
    ap.add_argument("--port", type=int, default=25010)
    ap.add_argument("--mem-util", type=float, default=0.5)
    ap.add_argument("--timeout", type=float, default=900.0)
    args = ap.parse_args(argv)
    name, arch_cfg = ARCHS[args.arch]
    args.model_dir = write_model_dir(os.path.join(tempfile.gettempdir(),
                                                  f"kvs_{args.arch}_dummy", name), arch_cfg)
    if args.compression == "controller":
        args.library = write_controller_library(
            os.path.join(tempfile.gettempdir(), f"kvs_library_{args.arch}.json"), name)
    if args.role != "both":
        return run_one_role(args)
    gpus = args.gpus.split(",")
    if len(gpus) != 2 * args.tp:
        raise SystemExit(f"--gpus needs {2 * args.tp} ids for --tp {args.tp}")
    gp, gc = ",".join(gpus[:args.tp]), ",".join(gpus[args.tp:])
    ctx = mp.get_context("spawn")
    qp, qc, qo = ctx.Queue(), ctx.Queue(), ctx.Queue()
    # each engine sees every GPU, its own first (peer mappings need both visible)
    pc = ctx.Process(target=engine, args=("c", f"{gc},{gp}", args, qc, qo))
    pp = ctx.Process(target=engine, args=("p", f"{gp},{gc}", args, qp, qo))
    pc.start()
    time.sleep(1.0)
    pp.start()
    deadline = time.time() + args.timeout
    ready = set()

    def get():
        left = deadline - time.time()
        if left <= 0:
            raise TimeoutError("engines did not answer in time")
        m = qo.get(timeout=left)
        if m[0] == "error":
            raise RuntimeError(f"engine {m[1]} failed:\n{m[2]}")
        return m

    rc = 0
    try:
        while len(ready) < 2:
            m = get()
            ready.add(m[1])
        ttft, prefill, first_tokens, agree = [], [], [], []
        vocab = ARCHS[args.arch][1]["vocab_size"]
        for i, ids in enumerate(prompts(args.warmup + args.requests, args.prompt_len, vocab,
                                        args.prompt_len_max)):
            t0 = time.time()
            qp.put(("go", i, ids))
            qc.put(("go", i, ids))
            got = {}
            while len(got) < 2:
                m = get()
                got[m[1]] = m
            if i >= args.warmup:
                ttft.append((got["c"][3] - t0) * 1e3)
                prefill.append((got["p"][3] - t0) * 1e3)
                first_tokens.append(got["c"][4])
                # the producer's token comes from its own full prefill (no
                # transfer): the consumer's must match it exactly for raw KV
                agree.append(got["c"][4][:1] == got["p"][4][:1])
        q = sorted(ttft)
        line = {"metric": f"p50 TTFT, 1P1D ({name} random-init, {args.prompt_len} prompt)",
                "overlap": os.environ.get("KVSERVE_OVERLAP_MODE", "off"), "tp": args.tp,
                "max_tokens": args.max_tokens,
                "impl": args.impl, "compression": args.compression,
                "transport": args.transport if args.impl == "ours" else "reference NcclTransport",
                "requests": args.requests, "prompt_len": args.prompt_len,
                "ttft_ms_p50": round(statistics.median(ttft), 2),
                "ttft_ms_p90": round(q[int(0.9 * (len(q) - 1))], 2),
                "ttft_ms_mean": round(statistics.mean(ttft), 2),
                "producer_prefill_ms_p50": round(statistics.median(prefill), 2),
                "handoff_ms_p50": round(statistics.median(
                    [a - b for a, b in zip(ttft, prefill)]), 2),
                "first_token_agreement": round(sum(agree) / len(agree), 4),
                "output_md5": hashlib.md5(json.dumps(first_tokens).encode()).hexdigest(),
                "data": "synthetic uniform token ids; random-init weights (load_format=dummy)",
                "timing": "host wall clock from dispatch to the consumer's first token"}
        stats = _stats_summary()
        if stats:
            line["stats"] = stats
        tl = timeline_breakdown(os.environ.get("KVSERVE_TIMELINE_PATH"), args.warmup)
        if tl:
            line["timeline_ms_p50"] = tl
        print(json.dumps(line), flush=True)
    except Exception as e:  # noqa: BLE001
        print(json.dumps({"impl": args.impl, "compression": args.compression,
                          "error": f"{type(e).__name__}: {e}"[-6000:]}), flush=True)
        rc = 1
    finally:
        for q in (qp, qc):
            q.put(("stop",))
        for p in (pp, pc):
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
    return rc


def timeline_breakdown(path, skip: int = 0):
    """Median durations of the connector's timeline markers (both engines
    append ``<tag> <epoch>`` lines to the same file): the producer's
    ``wait_for_save`` (P save_enter -> save_exit, compress + send) and the
    consumer's ``start_load_kv`` (D load_enter -> load_exit)."""
    if not path or not os.path.exists(path):
        return None
    spans: dict = {"P": [], "D": []}
    open_at: dict = {}
    with open(path) as f:
        for line in f:
            parts = line.split()
            if len(parts) != 3:
                continue
            side, tag, t = parts[0], parts[1], float(parts[2])
            if tag.endswith("_enter"):
                open_at[side] = t
            elif tag.endswith("_exit") and side in open_at:
                spans.setdefault(side, []).append((t - open_at.pop(side)) * 1e3)
    out = {}
    for side, name in (("P", "producer_wait_for_save"), ("D", "consumer_start_load_kv")):
        v = spans.get(side, [])
        v = [x for x in v if x > 0.05] or v  # steps without a transfer record ~0
        if v:
            out[name] = round(statistics.median(v), 3)
    return out or None


def prompts(n: int, prompt_len: int, vocab: int = QWEN25_7B["vocab_size"],
            prompt_len_max: int = 0) -> list:
    """The deterministic request sequence both sides generate on their own
    (lengths uniform in [prompt_len, prompt_len_max] when the latter is set)."""
    import random
    rng = random.Random(0)
    out = []
    for _ in range(n):
        t = rng.randint(prompt_len, prompt_len_max) if prompt_len_max > prompt_len else prompt_len
        out.append([rng.randrange(0, vocab) for _ in range(t)])
    return out


def run_one_role(args) -> int:
    """One engine on this host (cross-node PD, one role per node).  Both sides
    submit the same deterministic requests with the same transfer ids; the
    consumer's latency per request runs from its own submission to its first
    token, so it includes waiting for the producer's KV.  The consumer prints
    median latency and an md5 fingerprint of its outputs (compare it with a
    raw-KV run to catch silent corruption); the producer its prefill latency.
    Start the consumer first: its control socket must be listening."""
    role = "p" if args.role == "producer" else "c"
    ctx = mp.get_context("spawn")
    q_in, q_out = ctx.Queue(), ctx.Queue()
    proc = ctx.Process(target=engine, args=(role, args.gpus, args, q_in, q_out))
    proc.start()
    lat, outs, rc = [], [], 0
    try:
        m = q_out.get(timeout=args.timeout)
        if m[0] == "error":
            raise RuntimeError(m[2])
        vocab = ARCHS[args.arch][1]["vocab_size"]
        for i, ids in enumerate(prompts(args.warmup + args.requests, args.prompt_len, vocab,
                                        args.prompt_len_max)):
            t0 = time.time()
            q_in.put(("go", i, ids))
            m = q_out.get(timeout=args.timeout)
            if m[0] == "error":
                raise RuntimeError(m[2])
            if i >= args.warmup:
                lat.append((m[3] - t0) * 1e3)
                outs.append(m[4])
        print(json.dumps({"metric": "per-request latency, one PD role per node",
                          "role": args.role, "impl": args.impl,
                          "compression": args.compression, "requests": args.requests,
                          "latency_ms_p50": round(statistics.median(lat), 2),
                          "output_md5": hashlib.md5(json.dumps(outs).encode()).hexdigest(),
                          **({"stats": _stats_summary()} if _stats_summary() else {})}),
              flush=True)
    except Exception as e:  # noqa: BLE001
        print(json.dumps({"role": args.role, "error": f"{type(e).__name__}: {e}"[-4000:]}),
              flush=True)
        rc = 1
    finally:
        q_in.put(("stop",))
        proc.join(timeout=60)
        if proc.is_alive():
            proc.terminate()
    return rc


if __name__ == "__main__":
    sys.exit(main())
