#!/usr/bin/env python
"""KV-handoff benchmark: per-request prefill->decode KV transfer time.

Metric: "PD KV-transfer ms/request & p50 TTFT (Qwen2.5-7B,
8K prompt); compression ratio".  Config: Qwen2.5-7B KV shapes (28 layers,
4 KV heads, head_dim 128), 8192-token prompts, default compression mode,
synthetic N(0,1) KV with 3% outlier key channels x12 stored in a paged cache
(16-token blocks) at shuffled block ids.

Both arms run the same stages on the same workload: the default mode's
randomized Hadamard + hybrid min-max quantization (hybrid_ratio 0.8, levels
12/8 high, 6/4 low) with one byte per code and no entropy coder, the
transfer, and dequantization + inverse transform into the consumer's paged
cache.  That is the stage set the reference can run on this machine: its
entropy coders (nvCOMP ANS through CuPy, the LC library) are not installed.
This framework's own default path (4-bit codes + interleaved rANS) is timed
as well and reported under ``full_path``.

One step hands off ``--requests-per-step`` requests:

* N = 1: round trip on one GPU -- fused quantize of every (layer, request)
  item from the paged cache, [rANS encode, decode,] fused dequantize +
  inverse transform + scatter into a second paged cache;
* N >= 2 (torchrun, one rank per GPU): ranks [0, N/2) are producers, rank
  r + N/2 is r's consumer.  Each step is one message sent through the
  product path: ``FusedCompressionManager.send_paged_requests`` over the
  NVLink ring transport (``P2PTransport``), where the quantize kernel (byte
  codes) or the rANS compaction kernel stores straight into the consumer's
  receive ring and the last CTA publishes the ready flag; the consumer waits
  on the flag on the device, verifies the message checksum and decodes into
  its paged cache (``decompress_paged_requests``).

``value`` is ms per request of one producer/consumer pair (lower is
better): each rank times its stream with CUDA events between barriers, the
maximum over ranks is divided by the requests one pair handed off.  Per-pair
work is fixed as N grows (weak scaling), so equal values at every N mean
linear scaling.  ``e2e`` is the same path with every step's request
descriptors copied host->device from pinned memory and the step's result
(the device error word) read back.  At N >= 2 ``single_request_latency_ms``
is one un-pipelined request, from the producer's first kernel to the
consumer's scatter completing (the consumer's release flag lands back in
the producer's memory), device-timed on the producer.

``--impl reference`` runs the unmodified reference package from
``baseline/_ref``: its fused TileLang op ``KVHadamardQuantOp.compress_v3`` /
``decompress_v3`` per layer, in the order of its TileLang manager
(kvserve_v1/compression/tilelang_manager.py:158-216, :353-385) minus the
codec stage, its block extract/inject utilities, and at N >= 2 its wire
envelope and ``NcclTransport``.  ``decompress_v3`` imports
``fast_hadamard_transform`` (not installed); the arm supplies the plain
PyTorch stand-in in ``baseline/standin`` (one matrix product).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from typing import Optional

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "PD KV-transfer ms/request & p50 TTFT (Qwen2.5-7B, 8K prompt); compression ratio"
MODEL = "Qwen2.5-7B-Instruct"
HADAMARD_SEED = 0x3333  # the reference manager's default seed (manager.py:159)


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description="KV handoff benchmark")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--requests-per-step", type=int, default=8)
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--kv-heads", type=int, default=4)
    ap.add_argument("--block-size", type=int, default=16)
    ap.add_argument("--kv-layout", default="hnd", choices=["hnd", "nhd"],
                    help="paged block layout: hnd (head-major, vLLM FlashInfer on B200) or nhd")
    ap.add_argument("--codec", default="none", choices=["none", "rans", "bitpack"],
                    help="codec of the headline path (none: the stages both arms can run)")
    ap.add_argument("--no-full-path", action="store_true",
                    help="skip timing this framework's default path (4-bit codes + rANS)")
    ap.add_argument("--engine", default="tcgen05", choices=["tcgen05", "simt"])
    ap.add_argument("--compression", default="default", choices=["default", "off"],
                    help="off: raw KV blocks (no transform, quantization or codec)")
    ap.add_argument("--hybrid-ratio", type=float, default=None,
                    help="override the default mode's hybrid_ratio")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--latency-reps", type=int, default=5)
    ap.add_argument("--seed", type=int, default=0)
    return ap.parse_args(argv)


# ------------------------------------------------------------------ distributed
def dist_info():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def init_dist(world: int, local: int):
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def allreduce_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def allreduce_sum(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def first_non_none(x, world: int):
    """The value of the first rank that has one (all ranks call this)."""
    if world == 1:
        return x
    import torch.distributed as dist
    gathered = [None] * world
    dist.all_gather_object(gathered, x)
    return next((g for g in gathered if g is not None), None)


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons (200 ms)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = set(gpus)
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="kvs_clocks_", suffix=".csv")
            os.close(fd)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        sms, maxes, reasons, powers = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    idx = int(parts[0])
                except ValueError:
                    continue
                if idx not in self.gpus:
                    continue
                try:
                    sms.append(float(parts[1]))
                    maxes.append(float(parts[2]))
                    powers.append(float(parts[3]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.unlink(self.path)
        loaded = [s for s, p in zip(sms, powers) if p > 250] or sms
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(maxes) if maxes else None,
                "reasons": sorted(reasons), "samples": len(sms),
                "power_w_max": max(powers) if powers else None}


# ------------------------------------------------------------------ workload
def outlier_channels(num_heads: int, head_dim: int, fraction: float, seed: int) -> torch.Tensor:
    """Bool [H, D]: round(fraction * D) channels per head, drawn with a seeded
    CPU generator (the same workload for both arms, built without importing
    either framework)."""
    g = torch.Generator().manual_seed(seed)
    k = max(1, round(fraction * head_dim))
    mask = torch.zeros(num_heads, head_dim, dtype=torch.bool)
    for h in range(num_heads):
        mask[h, torch.randperm(head_dim, generator=g)[:k]] = True
    return mask


class Workload:
    """Source and destination paged caches for one rank."""

    def __init__(self, args, device, seed, role="both"):
        L, H, bs, T, B = args.layers, args.kv_heads, args.block_size, args.tokens, args.requests_per_step
        nb = (T + bs - 1) // bs
        self.nblocks = B * nb + 7
        self.L, self.H, self.bs, self.T, self.B, self.nb = L, H, bs, T, B, nb
        g = torch.Generator(device="cpu").manual_seed(seed)
        perm_src = torch.randperm(self.nblocks, generator=g).tolist()
        perm_dst = torch.randperm(self.nblocks, generator=g).tolist()
        self.src_req = [(perm_src[i * nb:(i + 1) * nb], T) for i in range(B)]
        self.dst_req = [(perm_dst[i * nb:(i + 1) * nb], T) for i in range(B)]
        self.layout = getattr(args, "kv_layout", "hnd")
        self.src = self.dst = None
        if role in ("both", "producer"):
            self.src = self._alloc(L, H, bs, device, zero=False)
            gd = torch.Generator(device=device).manual_seed(seed + 17)
            for l in range(L):  # fill layer by layer to bound temporaries
                self.src[l].normal_(generator=gd)
            m = outlier_channels(H, 128, fraction=0.03, seed=seed + 3).to(device)
            scale = torch.where(m, 12.0, 1.0).to(torch.bfloat16)
            for l in range(L):
                self.src[l, 0].mul_(scale)  # [nb, bs, H, D] * [H, D]
        if role in ("both", "consumer"):
            self.dst = self._alloc(L, H, bs, device, zero=True)

    def _alloc(self, L, H, bs, device, zero):
        """Logical [L, 2, nblocks, bs, H, D] paged caches.  HND: each block
        stores its heads one after another (head-major), the layout vLLM's
        FlashInfer backend allocates on B200; NHD: token-major blocks."""
        make = torch.zeros if zero else torch.empty
        if self.layout == "hnd":
            t = make((L, 2, self.nblocks, H, bs, 128), dtype=torch.bfloat16, device=device)
            return t.permute(0, 1, 2, 4, 3, 5)
        return make((L, 2, self.nblocks, bs, H, 128), dtype=torch.bfloat16, device=device)

    @property
    def bf16_bytes_per_request(self) -> int:
        return self.L * 2 * self.T * self.H * 128 * 2

    def src_layers(self):
        return [self.src[l] for l in range(self.L)]

    def dst_layers(self):
        return [self.dst[l] for l in range(self.L)]


def quant_config(args, codec=None):
    from kvserve_hpdps_b200.compression.config import get_default_compression_config
    cfg = get_default_compression_config()
    cfg["quantizer_config"]["model_name"] = MODEL
    if getattr(args, "hybrid_ratio", None) is not None:
        cfg["quantizer_config"]["hybrid_ratio"] = float(args.hybrid_ratio)
    codec = codec or args.codec
    if codec == "bitpack":
        cfg["codec_config"] = {"codec_type": "bitpack"}
    elif codec == "none":
        cfg["codec_config"] = {"codec_type": "none"}
    return cfg


# the default mode's quantizer in both frameworks (hybrid ratio, high key /
# value levels, low key / value levels)
DEFAULT_QUANTIZER = {"hybrid_ratio": 0.8, "high_key_max_value": 12, "high_value_max_value": 8,
                     "low_key_max_value": 6, "low_value_max_value": 4}


def hybrid_ratio(args) -> float:
    hr = getattr(args, "hybrid_ratio", None)
    return float(hr) if hr is not None else DEFAULT_QUANTIZER["hybrid_ratio"]


def compression_label(args, codec=None) -> str:
    """The ``config.compression`` string: identical for both arms."""
    if args.compression == "off":
        return "off (raw bf16 blocks)"
    codec = codec or args.codec
    codes = {"none": "u8 codes, no entropy codec", "rans": "4-bit codes + rANS",
             "bitpack": "bit-packed codes"}[codec]
    return f"default mode: Hadamard + hybrid {hybrid_ratio(args)} 12/8/6/4, {codes}"


def _roles(world, rank):
    pairs = max(1, world // 2)
    if world == 1:
        return "both", pairs
    if world % 2:
        raise SystemExit("--gpus must be 1 or even")
    return ("producer" if rank < pairs else "consumer"), pairs


def side_port(offset, pair_id):
    return int(os.environ.get("MASTER_PORT", "29500")) + offset + pair_id


def _events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def _timed_loop(step, s0: int, steps: int, world: int, device, side_streams=()):
    """``steps`` steps between a barrier + device synchronisation on both
    sides, timed with CUDA events on the current stream (work a step queues
    on ``side_streams`` starts after the first event and is joined before the
    second); returns (max ms over ranks, next step index)."""
    barrier(world)
    torch.cuda.synchronize(device)
    main = torch.cuda.current_stream(device)
    ev0, ev1 = _events()
    ev0.record()
    for st in side_streams:
        st.wait_stream(main)
    s = s0
    for _ in range(steps):
        step(s)
        s += 1
    for st in side_streams:
        main.wait_stream(st)
    ev1.record()
    torch.cuda.synchronize(device)
    barrier(world)
    return allreduce_max(ev0.elapsed_time(ev1), world), s


def _poll_message(tr, pending, key, timeout_s):
    """Wait (bounded) until the transport delivered the message ``key``."""
    deadline = time.monotonic() + timeout_s
    while key not in pending or not pending[key]:
        for k, v in tr.drain_received().items():
            pending.setdefault(k, []).extend(v)
        if key in pending and pending[key]:
            break
        if time.monotonic() > deadline:
            raise TimeoutError(f"message {key} did not arrive within {timeout_s} s")
        waiter = getattr(tr, "wait_received", None)
        if waiter is not None:
            waiter(0.0005)
        else:
            time.sleep(2e-5)
    return pending[key].pop(0)


# ------------------------------------------------------------------ ours
def make_manager(args, codec):
    from kvserve_hpdps_b200.compression.fused_manager import FusedCompressionManager
    cfg = quant_config(args, codec)
    engine = 1 if args.engine == "simt" else 0
    return FusedCompressionManager(args.kv_heads, 128, cfg["quantizer_config"],
                                   cfg["codec_config"], base_seed=HADAMARD_SEED, engine=engine)


def run_ours_raw(args, rank, world, local, wl):
    """Compression off: raw KV blocks.  N = 1: one gather launch of every
    (layer, request) item from the paged cache into a flat buffer and one
    scatter launch into the second cache.  N >= 2: through the ring
    transport's ``send_paged`` (one gather launch storing straight into the
    consumer's ring, checksum and ready flag included); the consumer scatters
    with one launch."""
    from kvserve_hpdps_b200.ops import kernels as K
    device = torch.device("cuda", local)
    role, pairs = _roles(world, rank)
    pair_id = rank % pairs
    L = args.layers
    if world == 1:
        src_raw = K.RawItems(wl.src_layers(), [(l, b) for b, _ in wl.src_req for l in range(L)])
        dst_raw = K.RawItems(wl.dst_layers(), [(l, b) for b, _ in wl.dst_req for l in range(L)])
        flat = torch.empty(src_raw.flat_bytes, dtype=torch.uint8, device=device)

        def step(s):
            K.paged_raw(src_raw, flat.data_ptr(), True)
            K.paged_raw(dst_raw, flat.data_ptr(), False)
        launches, transport = 2, "local"
    else:
        tr = _open_transport(args, role, pair_id, device, wl.bf16_bytes_per_request * wl.B)
        names = [f"model.layers.{l}.self_attn.attn" for l in range(L)]
        pending: dict = {}
        blocks_all = [b for blocks, _ in wl.src_req for b in blocks]
        dst_all = [b for blocks, _ in wl.dst_req for b in blocks] if wl.dst is not None else None

        def step(s):
            if role == "producer":
                tr.send_paged(f"s{s}", names, wl.src_layers(), blocks_all)
            else:
                _, payload = _poll_message(tr, pending, f"s{s}", 60.0)
                tr.prepare(payload, device)
                dst_raw = K.RawItems(wl.dst_layers(), [(l, dst_all) for l in range(L)])
                K.paged_raw(dst_raw, payload["tensor"].data_ptr(), False)
                tr.release(payload, device)
        launches = 1 if role == "producer" else 4
        transport = "nvlink-p2p ring (P2PTransport.send_paged: one gather launch stores raw " \
                    "blocks into the consumer's ring)"
    s = 0
    for _ in range(args.warmup):
        step(s)
        s += 1
    torch.cuda.synchronize(device)
    sampler = ClockSampler(range(world)) if local == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    ms, s = _timed_loop(step, s, args.steps, world, device)
    clocks = sampler.stop() if sampler else None
    err = int(allreduce_max(float(K.read_device_error(device)), world))
    error = None
    if role in ("both", "consumer"):
        ref = wl if wl.src is not None else Workload(args, device, args.seed + 101 * pair_id,
                                                     "producer")
        idx_s = torch.tensor(ref.src_req[0][0], device=device)
        idx_d = torch.tensor(wl.dst_req[0][0], device=device)
        error = {"exact": bool(torch.equal(ref.src[:, :, idx_s], wl.dst[:, :, idx_d]))}
        del ref
    error = first_non_none(error, world)
    if world > 1:
        if role == "producer":
            tr.wait_for_sent(60.0)
        barrier(world)
        tr.close()
    return {"ms": ms, "cr": 1.0, "error": error, "transport": transport,
            "launches": launches * args.steps, "clocks": clocks, "device_error": err,
            "pairs": pairs, "role": role}


def _open_transport(args, role, pair_id, device, message_bytes: int):
    from kvserve_hpdps_b200.parallel.p2p_transport import P2PTransport
    ring = int(os.environ.get("KVSERVE_RING_BYTES", str(max(2 << 30, int(3.2 * message_bytes)))))
    return P2PTransport(role == "producer", "127.0.0.1", side_port(600, pair_id), device.index, 0,
                        ring_bytes=ring, n_flags=256)


def run_path(args, mgr, wl, rank, world, local, e2e: bool, latency: bool, clocks: bool):
    """Time one codec path of this framework (headline or full path)."""
    listener = _SizeListener()
    from kvserve_hpdps_b200.ops import kernels as K
    device = torch.device("cuda", local)
    role, pairs = _roles(world, rank)
    pair_id = rank % pairs
    L = args.layers
    engine = mgr.engine
    use_rans = mgr.stream_codec == "rans"
    plans = [mgr.plan(l) for l in range(L)]
    out = {"pairs": pairs, "role": role}
    sampler = None
    if world == 1:
        src_slots = K.LayerSlots(wl.src_layers(), plans)
        dst_slots = K.LayerSlots(wl.dst_layers(), plans)
        src_items = K.WorkItems(src_slots, [(l, b, n) for l in range(L) for b, n in wl.src_req])
        dst_items = K.WorkItems(dst_slots, [(l, b, n) for l in range(L) for b, n in wl.dst_req])
        code_bytes, meta_bytes = src_items.code_bytes, src_items.meta_bytes
        codes = torch.empty(code_bytes, dtype=torch.uint8, device=device)
        meta = torch.empty(meta_bytes, dtype=torch.uint8, device=device)
        cap = K.rans_max_bytes(code_bytes) if use_rans else code_bytes
        stream_buf = torch.empty(cap, dtype=torch.uint8, device=device) if use_rans else None
        dec_codes = torch.empty(code_bytes, dtype=torch.uint8, device=device) if use_rans else codes

        def compress(s):
            K.quantize(src_slots, src_items, codes, meta, engine=engine)
            if use_rans:
                K.rans_encode_ptr(codes.data_ptr(), code_bytes, stream_buf.data_ptr(), device)

        def decompress(s):
            if use_rans:
                K.rans_decode_ptr(stream_buf.data_ptr(), code_bytes, dec_codes.data_ptr(), device,
                                  stream_bytes=cap)
            K.dequantize(dec_codes, meta, dst_slots, dst_items, engine=engine)

        def step(s):
            compress(s)
            decompress(s)
        launches = 4 + (4 if use_rans else 0) + 1
        out["transport"] = "local"
        s = 0
        for _ in range(args.warmup):
            step(s)
            s += 1
        torch.cuda.synchronize(device)
        K.check_device_error(device, "warm-up")
        if use_rans:
            stream_bytes = K.rans_encode(codes, out=torch.empty_like(stream_buf)).numel() + 16
        else:
            stream_bytes = code_bytes
        out["wire_bytes_per_step"] = stream_bytes + meta_bytes
        out["error"] = K.kv_error(wl.src[:, :, torch.tensor(wl.src_req[0][0], device=device)],
                                  wl.dst[:, :, torch.tensor(wl.dst_req[0][0], device=device)])
        if clocks:
            sampler = ClockSampler([local])
            sampler.start()
            time.sleep(0.3)
        out["ms"], s = _timed_loop(step, s, args.steps, world, device)
        if sampler:
            out["clocks"] = sampler.stop()
        out["launches"] = launches * args.steps
        ms_c, s = _timed_loop(compress, s, args.steps, world, device)
        ms_d, s = _timed_loop(decompress, s, args.steps, world, device)
        n = args.steps * wl.B
        out["stage_ms_per_request"] = {"compress": round(ms_c / n, 5),
                                       "decompress": round(ms_d / n, 5)}
        out["device_error"] = K.read_device_error(device)
        if e2e:
            out["e2e"] = _e2e_local(args, mgr, wl, device)
        return out

    # ---------------- N >= 2: producer/consumer pairs over the ring transport
    from kvserve_hpdps_b200.compression.manager import add_sentinel
    from kvserve_hpdps_b200.compression.wire import CompressedWire, restore_from_wire
    from kvserve_hpdps_b200.parallel.p2p import DeviceRegion, PeerMapping
    tr = _open_transport(args, role, pair_id, device, wl.bf16_bytes_per_request * wl.B)
    if role == "producer":  # exact bytes on the link of each sent message
        tr.add_sent_listener(listener)
    names = add_sentinel([f"model.layers.{l}.self_attn.attn" for l in range(L)])
    pending: dict = {}
    # producer-owned release flags, written by its consumer (single-request latency)
    region = DeviceRegion(local, 4096)
    handles = [None] * world
    import torch.distributed as dist
    dist.all_gather_object(handles, (region.ipc_handle(), region.nbytes))
    peer = rank + pairs if role == "producer" else rank - pairs
    peer_map = PeerMapping(local, handles[peer][0], handles[peer][1])
    sizes = []

    def produce(s, reqs, tids):
        info = mgr.send_paged_requests(tr, f"s{s}", names, wl.src_layers(), list(range(L)), reqs,
                                       member_tids=tids)
        sizes.append(info["wire_nbytes"])

    def consume(s, reqs):
        _, payload = _poll_message(tr, pending, f"s{s}", 60.0)
        tr.prepare(payload, device)
        cd = restore_from_wire(CompressedWire(payload["meta"], payload["body_chunks"],
                                              payload["aux_tensors"]))
        mgr.decompress_paged_requests(cd, wl.dst_layers(), reqs)
        tr.release(payload, device)

    # Consecutive messages of a producer alternate between two streams: the
    # statistics pass of message s+1 (HBM-bound) runs while message s's
    # quantize kernel stores over NVLink (link-bound).  Kernel scratch is per
    # stream, and the ring transport orders nothing by stream.
    prod_streams = [torch.cuda.Stream(device), torch.cuda.Stream(device)] \
        if role == "producer" else []

    def step(s):
        if role == "producer":
            with torch.cuda.stream(prod_streams[s % 2]):
                produce(s, wl.src_req, [f"{s}:{r}" for r in range(wl.B)])
        else:
            consume(s, wl.dst_req)
    out["transport"] = ("nvlink-p2p ring: FusedCompressionManager.send_paged_requests -> "
                        "P2PTransport.open_message/commit_message; quantize "
                        + ("-> rANS compaction kernel" if use_rans else "kernel")
                        + " stores into the consumer's ring, last CTA publishes the flag")
    s = 0
    for _ in range(args.warmup):
        step(s)
        s += 1
    if role == "producer":
        tr.wait_for_sent(120.0)
    torch.cuda.synchronize(device)
    barrier(world)
    err = K.read_device_error(device)
    if err:
        raise RuntimeError(f"device error {err} during warm-up ({K.ERR_NAMES.get(err)})")
    error = None
    if role == "consumer":
        ref = Workload(args, device, args.seed + 101 * pair_id, "producer")
        error = K.kv_error(ref.src[:, :, torch.tensor(ref.src_req[0][0], device=device)],
                           wl.dst[:, :, torch.tensor(wl.dst_req[0][0], device=device)])
        del ref
        torch.cuda.empty_cache()
    out["error"] = first_non_none(error, world)
    if clocks and local == 0:
        sampler = ClockSampler(range(world))
        sampler.start()
        time.sleep(0.3)

    out["ms"], s = _timed_loop(step, s, args.steps, world, device, side_streams=prod_streams)
    if sampler:
        out["clocks"] = sampler.stop()
    if role == "producer":
        tr.wait_for_sent(120.0)
    # wire bytes: the exact coded sizes come back through the transport's listeners
    launches = (7 + (4 if use_rans else 0)) if role == "producer" else 6
    out["launches"] = launches * args.steps
    out["device_error"] = int(allreduce_max(float(K.read_device_error(device)), world))

    if latency and args.latency_reps > 0:
        lat = []
        for i in range(args.latency_reps):
            tag = 1000 + i
            barrier(world)
            torch.cuda.synchronize(device)
            if role == "producer":
                ev0, ev1 = _events()
                ev0.record()
                produce(f"lat{i}", wl.src_req[:1], [f"lat{i}"])
                K.wait_flag(region.ptr, tag, device, timeout_s=20.0)
                ev1.record()
                torch.cuda.synchronize(device)
                lat.append(ev0.elapsed_time(ev1))
            else:
                consume(f"lat{i}", wl.dst_req[:1])
                K.set_flag(peer_map.ptr, tag, device)
                torch.cuda.synchronize(device)
        med = statistics.median(lat) if lat else 0.0
        out["single_request_latency_ms"] = round(allreduce_max(med, world), 4)
        if K.read_device_error(device):
            raise RuntimeError("device error during the latency probe")
    if e2e:
        out["e2e"] = _e2e_pairs(args, mgr, wl, tr, role, world, pairs, device, names, pending)
    if role == "producer":
        tr.wait_for_sent(120.0)
    out["wire_bytes_per_step"] = statistics.median(listener.sizes) if listener.sizes else None
    out["ring_reserved_bytes_per_step"] = statistics.median(sizes) if sizes else None
    barrier(world)
    tr.close()
    peer_map.close()
    barrier(world)
    region.close()
    return out


def _e2e_local(args, mgr, wl, device):
    """N = 1 through the public manager API: every step builds the request
    descriptors on the host and copies them host->device from pinned memory
    (inside compress/decompress_paged_requests), compresses into one wire
    message and decodes it into the consumer cache, then reads the device
    error word back (the step's result)."""
    from kvserve_hpdps_b200.ops import kernels as K
    L = wl.L
    steps = max(2, min(args.steps, 10))

    errs = K.StepErrors(device)

    def one():
        cd = mgr.compress_paged_requests(wl.src_layers(), list(range(L)), wl.src_req, trim=False)
        mgr.decompress_paged_requests(cd, wl.dst_layers(), wl.dst_req)
        errs.push()  # this step's error word to pinned host memory
        errs.check(keep=1)  # the previous step's word, read while this step runs
    for _ in range(2):
        one()
    errs.check(0)
    torch.cuda.synchronize(device)
    K.reset_transfer_counters()
    ev0, ev1 = _events()
    ev0.record()
    for _ in range(steps):
        one()
    errs.check(0)  # the last step's result
    ev1.record()
    torch.cuda.synchronize(device)
    c = K.transfer_counters()
    return {"value": round(ev0.elapsed_time(ev1) / (steps * wl.B), 5), "unit": "ms/request",
            "h2d_bytes_per_step": c["h2d"] // steps, "d2h_bytes_per_step": c["d2h"] // steps,
            "steps": steps,
            "path": "compress_paged_requests -> decompress_paged_requests; each step's error "
                    "word copied to pinned host memory and read while the next step runs"}


def _e2e_pairs(args, mgr, wl, tr, role, world, pairs, device, names, pending):
    """N >= 2 through the public API, as the connector drives it: the
    producer's ``send_paged_requests`` (descriptors host->device from pinned
    memory, kernels storing into the consumer's ring), the consumer's drain
    -> ``prepare`` (bounded flag wait, checksum) -> ``restore_from_wire`` ->
    ``decompress_paged_requests``; every step both ranks read their device
    error word back."""
    from kvserve_hpdps_b200.compression.wire import CompressedWire, restore_from_wire
    from kvserve_hpdps_b200.ops import kernels as K
    L = wl.L
    steps = max(2, min(args.steps, 10))

    errs = K.StepErrors(device)

    def one(s):
        if role == "producer":
            mgr.send_paged_requests(tr, f"e{s}", names, wl.src_layers(), list(range(L)),
                                    wl.src_req, member_tids=[f"e{s}:{r}" for r in range(wl.B)])
        else:
            _, payload = _poll_message(tr, pending, f"e{s}", 60.0)
            tr.prepare(payload, device)
            cd = restore_from_wire(CompressedWire(payload["meta"], payload["body_chunks"],
                                                  payload["aux_tensors"]))
            mgr.decompress_paged_requests(cd, wl.dst_layers(), wl.dst_req)
            tr.release(payload, device)
        errs.push()  # this step's error word to pinned host memory
        errs.check(keep=1)  # the previous step's word, read while this step runs
    s = 0
    for _ in range(2):
        one(s)
        s += 1
    errs.check(0)
    if role == "producer":
        tr.wait_for_sent(120.0)
    torch.cuda.synchronize(device)
    barrier(world)
    K.reset_transfer_counters()
    ev0, ev1 = _events()
    ev0.record()
    for _ in range(steps):
        one(s)
        s += 1
    errs.check(0)  # the last step's result
    if role == "producer" and not tr.wait_for_sent(120.0):
        raise TimeoutError("sends did not complete")
    ev1.record()
    torch.cuda.synchronize(device)
    ms = allreduce_max(ev0.elapsed_time(ev1), world)
    c = K.transfer_counters()
    h2d = allreduce_sum(float(c["h2d"]), world) / (steps * pairs)
    d2h = allreduce_sum(float(c["d2h"]), world) / (steps * pairs)
    return {"value": round(ms / (steps * wl.B), 5), "unit": "ms/request",
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": steps,
            "path": "send_paged_requests -> P2PTransport ring -> drain_received/prepare -> "
                    "restore_from_wire -> decompress_paged_requests; each step's error word "
                    "copied to pinned host memory and read while the next step runs"}


class _SizeListener:
    """Exact coded bytes of each sent message (the transport's completion thread)."""

    def __init__(self):
        self.sizes = []

    def __call__(self, request_id, tids, ms, nbytes=None):
        if nbytes is not None and not str(request_id).startswith(("lat", "e")):
            self.sizes.append(int(nbytes))


def run_ours(args, rank, world, local):
    device = torch.device("cuda", local)
    role, pairs = _roles(world, rank)
    pair_id = rank % pairs
    wl = Workload(args, device, args.seed + 101 * pair_id, role)
    if args.compression == "off":
        return run_ours_raw(args, rank, world, local, wl)
    paths = [(args.codec, True)]
    if not args.no_full_path and args.codec != "rans":
        paths.append(("rans", False))
    results = []
    for codec, headline in paths:
        mgr = make_manager(args, codec)
        res = run_path(args, mgr, wl, rank, world, local, e2e=not args.no_e2e,
                       latency=world > 1, clocks=headline)
        torch.cuda.synchronize(device)
        results.append((codec, res))
        torch.cuda.empty_cache()
    head = results[0][1]
    head["codec"] = results[0][0]
    for codec, res in results[1:]:
        head["full_path"] = _summary(args, wl, res, world, codec)
    head["cr"] = _cr(args, wl, head, world)
    head["launches_total"] = head["launches"] + sum(r["launches"] for _, r in results[1:])
    return head


def _cr(args, wl, res, world):
    """Whole-job compression ratio: raw bytes over the bytes on the wire."""
    b = res.get("wire_bytes_per_step")
    tot = allreduce_sum(float(b or 0), world) if world > 1 else float(b or 0)
    n_prod = res["pairs"] if world > 1 else 1
    orig = wl.bf16_bytes_per_request * wl.B * n_prod
    return orig / tot if tot else None


LINK_GBS = 770.0  # measured NVLink 5 peer copy per direction on this pool's B200s


def _peaks() -> tuple[float, str]:
    """HBM copy bandwidth (read + write bytes): MEASURED_PEAKS.json when the
    driver wrote it, else the earlier measurement of this pool."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, ValueError, KeyError):
        return 6650.0, "fallback"


def roofline(args, world: int, codec: str, cr: Optional[float], ms: float) -> dict:
    """The path's roofline per request: the slower of its algorithmic HBM
    bytes at the copy bandwidth and its bytes over NVLink at the peer-copy
    bandwidth, and the measured time's fraction of it.  The key statistics
    span every token of a request-layer, so the input is read twice (a
    statistics pass, then quantization); codes are one byte (``none``),
    4-bit nibbles (``rans``) or the bit-packed wire bytes (``bitpack``);
    the rANS codes make a round trip through HBM on each side (written by
    the quantize kernel, read by the encoder; written by the decoder, read
    by the dequantize kernel)."""
    raw = args.layers * 2 * args.tokens * args.kv_heads * 128 * 2
    wire = raw / cr if cr else None
    codes = {"none": raw / 2, "rans": raw / 4}.get(codec, wire or raw / 2)
    stream = wire if codec == "rans" and wire else codes
    hbm, src = _peaks()
    # the message (codes, or the rANS stream) is written once into the
    # consumer's memory: over NVLink at N >= 2, into the same HBM at N = 1
    msg = stream if codec == "rans" else codes
    local = 2 * codes if codec == "rans" else 0  # codes' round trip on each side
    prod = 2 * raw + local
    cons = msg + msg + local + raw  # written by the producer, read, decoded, scattered
    if world == 1:  # one GPU does both halves; nothing crosses NVLink
        parts = {"hbm": (prod + cons) / hbm}
    else:  # producer and consumer run side by side, each message pipelined
        parts = {"hbm-producer": prod / hbm, "nvlink": msg / LINK_GBS,
                 "hbm-consumer": cons / hbm}
    parts = {k: v / 1e6 for k, v in parts.items()}  # GB/s -> ms per request
    bound = max(parts, key=parts.get)
    return {"bound_ms": round(parts[bound], 5), "limited_by": bound,
            "fraction": round(parts[bound] / ms, 3) if ms > 0 else None,
            "terms_ms": {k: round(v, 5) for k, v in parts.items()},
            "hbm_gbs": hbm, "link_gbs": LINK_GBS, "peaks": src}


def _summary(args, wl, res, world, codec):
    ms = res["ms"] / (args.steps * wl.B)
    out = {"compression": compression_label(args, codec), "value": round(ms, 5),
           "unit": "ms/request", "compression_ratio": None,
           "reconstruction": res.get("error"), "launches": res["launches"]}
    cr = _cr(args, wl, res, world)
    out["compression_ratio"] = round(cr, 3) if cr else None
    out["roofline"] = roofline(args, world, codec, cr, ms)
    for k in ("e2e", "stage_ms_per_request", "single_request_latency_ms"):
        if res.get(k) is not None:
            out[k] = res[k]
    return out


# ------------------------------------------------------------------ reference
_REF_TRANSPORTS: dict = {}


def _ref_imports():
    """Put the reference install and the fast_hadamard_transform stand-in on
    sys.path; nothing of this repository's package is imported on this arm."""
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    standin = os.path.join(ROOT, "baseline", "standin")
    for p in (standin, ref_root):
        if p not in sys.path:
            sys.path.insert(0, p)


class _RefPipeline:
    """The reference's fused op driven as its TileLang manager does
    (kvserve_v1/compression/tilelang_manager.py:158-216 and :353-385), with
    the codec stage left out: per layer ``compress_v3`` then the heads-outer
    permute and ``_canon_meta``; on the way back ``_decanon_meta``, the
    inverse permute and ``decompress_v3`` per layer."""

    def __init__(self, args):
        from kvserve_v1.compression.compression_manager import CompressedKVData
        from kvserve_v1.compression.tilelang_manager import _canon_meta, _decanon_meta
        from kvserve_v1.tilelang_ops.kv_hadamard_quant import KVHadamardQuantOp
        qc = dict(DEFAULT_QUANTIZER, model_name=MODEL, hybrid_ratio=hybrid_ratio(args))
        self.op = KVHadamardQuantOp(num_heads=args.kv_heads, head_dim=128, base_seed=HADAMARD_SEED,
                                    dtype=torch.bfloat16, quant_type="minmax",
                                    axis_key="channel", axis_value="token", split_type="head",
                                    **qc)
        self.CompressedKVData = CompressedKVData
        self._canon, self._decanon = _canon_meta, _decanon_meta

    def compress(self, stacked: torch.Tensor, request_id: str):
        L = stacked.shape[0]
        q_layers, qparams = [], []
        for l in range(L):
            q, m = self.op.compress_v3(stacked[l].contiguous(), layer_id=l)
            q_layers.append(q.permute(0, 3, 1, 2, 4).contiguous())
            qparams.append(self._canon(m))
        buffer = torch.stack(q_layers, dim=0).contiguous()
        meta = {"request_id": request_id, "num_layers": L, "codec_applied": False,
                "codec_shape": list(buffer.shape), "codec_dtype": "uint8",
                "device": str(buffer.device), "original_dtype": "bfloat16",
                "original_shape": list(stacked.shape), "quantization_params": qparams,
                "backend": "tilelang_v3"}
        return self.CompressedKVData(request_id=request_id, layer_id=L - 1,
                                     compressed_tensor=buffer, metadata=meta,
                                     original_size=stacked.numel() * stacked.element_size(),
                                     compressed_size=buffer.numel() * buffer.element_size())

    def decompress(self, c) -> torch.Tensor:
        meta = c.metadata
        buffer = c.compressed_tensor.view(torch.uint8).reshape(meta["codec_shape"])
        outs = []
        for l in range(int(meta["num_layers"])):
            layer_q = buffer[l].permute(0, 2, 3, 1, 4).contiguous()
            outs.append(self.op.decompress_v3(layer_q, self._decanon(meta["quantization_params"][l]),
                                              layer_id=l))
        return torch.stack(outs, dim=0)


def _ref_error(src_wl, dst_wl, device):
    a = src_wl.src[:, :, torch.tensor(src_wl.src_req[0][0], device=device)].float()
    b = dst_wl.dst[:, :, torch.tensor(dst_wl.dst_req[0][0], device=device)].float()
    return {"cosine": float(torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0)),
            "rel_mse": float(((a - b) ** 2).sum() / (a ** 2).sum())}


REF_PIPELINE = ("reference KVHadamardQuantOp.compress_v3 / decompress_v3 per layer (TileLang "
                "kernels), in its TileLang manager's order without the codec stage (nvCOMP/CuPy "
                "and LC not installed); fast_hadamard_transform not installed: plain-PyTorch "
                "stand-in (baseline/standin); its extract/inject block utilities")


def _ref_e2e(args, world, device, step, s0: int, read_cache, read_blocks, h2d_per_step: int,
             pairs: int, finish=None) -> dict:
    """End to end through the reference's public API: the same step as the
    device-timed loop (its extract/inject utilities build their block-index
    tensors on the device from host lists every call; those copies are the
    step's host->device bytes), then the step's result read back: 4 bytes of
    the cache it wrote (a pinned, synchronous device->host copy, as the
    reference reads its results).  Every rank runs the same steps and reaches
    the same collectives whether or not its loop failed."""
    steps = max(2, min(args.steps, 10))
    host = torch.empty(2, dtype=torch.bfloat16, pin_memory=True)
    ms, err = -1.0, None
    try:
        barrier(world)
        torch.cuda.synchronize(device)
        ev0, ev1 = _events()
        ev0.record()
        s = s0
        for _ in range(steps):
            step(s)
            host.copy_(read_cache[:, read_blocks[0]].reshape(-1)[:2])  # the step's result
            s += 1
        if finish is not None:
            finish()
        ev1.record()
        torch.cuda.synchronize(device)
        ms = ev0.elapsed_time(ev1)
    except Exception as e:  # noqa: BLE001
        err = f"{type(e).__name__}: {e}"
    worst = allreduce_max(ms, world)
    failed = allreduce_max(1.0 if err else 0.0, world)
    if failed:
        return {"unavailable": err or "failed on another rank"}
    return {"value": round(worst / (steps * args.requests_per_step), 5), "unit": "ms/request",
            "h2d_bytes_per_step": int(h2d_per_step), "d2h_bytes_per_step": 4 * (world // pairs),
            "steps": steps,
            "path": "the reference's extract_kv_from_layer_by_blocks -> compress_v3 per layer"
                    + (" -> build_wire -> NcclTransport -> restore_from_wire" if world > 1
                       else "") + " -> decompress_v3 per layer -> "
                    "inject_kv_into_layer_by_blocks; each step's result read back"}


def run_reference(args, rank, world, local):
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "kvserve_v1")):
        return {"unavailable": "reference not installed in baseline/_ref"}
    _ref_imports()
    if world > 1:
        return run_reference_pairs(args, rank, world, local)
    from kvserve_v1.utils.kv_utils import (extract_kv_from_layer_by_blocks,  # noqa: E402
                                           inject_kv_into_layer_by_blocks)
    device = torch.device("cuda", local)
    raw = args.compression == "off"
    pipe = None if raw else _RefPipeline(args)
    wl = Workload(args, device, args.seed)
    L = args.layers
    sizes = []

    def extract(r):
        return torch.stack([extract_kv_from_layer_by_blocks(wl.src[l], wl.src_req[r][0])
                            for l in range(L)], dim=0)

    def inject(r, out):
        for l in range(L):
            inject_kv_into_layer_by_blocks(wl.dst[l], out[l], wl.dst_req[r][0])

    def step(s):
        for r in range(wl.B):
            stacked = extract(r)
            if raw:
                sizes.append(int(stacked.numel() * stacked.element_size()))
                out = stacked
            else:
                c = pipe.compress(stacked, f"r{s}_{r}")
                sizes.append(int(c.compressed_size) + _aux_bytes(c.metadata))
                out = pipe.decompress(c)
            inject(r, out)

    def compress_only(s):
        for r in range(wl.B):
            pipe.compress(extract(r), f"c{s}_{r}")

    s = 0
    for _ in range(args.warmup):
        step(s)
        s += 1
    torch.cuda.synchronize(device)
    sampler = ClockSampler([local])
    sampler.start()
    time.sleep(0.3)
    ms, s = _timed_loop(step, s, args.steps, world, device)
    clocks = sampler.stop()
    out = {"ms": ms, "error": _ref_error(wl, wl, device), "clocks": clocks,
           "pipeline": "raw: extract_kv_from_layer_by_blocks + stack + "
                       "inject_kv_into_layer_by_blocks" if raw else REF_PIPELINE,
           "transport": "local", "pairs": 1}
    out["cr"] = wl.bf16_bytes_per_request / statistics.mean(sizes[-args.steps * wl.B:])
    if not raw:
        ms_c, s = _timed_loop(compress_only, s, args.steps, world, device)
        n = args.steps * wl.B
        out["stage_ms_per_request"] = {"compress": round(ms_c / n, 5),
                                       "decompress": round((ms - ms_c) / n, 5)}
    if not args.no_e2e:
        nb = len(wl.src_req[0][0])
        out["e2e"] = _ref_e2e(args, world, device, step, s, wl.dst[L - 1], wl.dst_req[-1][0],
                              wl.B * L * 2 * nb * 8, 1)
    return out


def _aux_bytes(meta) -> int:
    """Bytes of the tensors in a message's quantization parameters (the
    metadata that travels next to the codes)."""
    tot = 0

    def walk(x):
        nonlocal tot
        if isinstance(x, torch.Tensor):
            tot += x.numel() * x.element_size()
        elif isinstance(x, dict):
            for v in x.values():
                walk(v)
        elif isinstance(x, (list, tuple)):
            for v in x:
                walk(v)
    walk(meta.get("quantization_params"))
    return tot


def run_reference_pairs(args, rank, world, local):
    """Reference arm on producer/consumer pairs, through the reference's own
    public modules: the fused op pipeline above, its wire envelope
    (build_wire / restore_from_wire), its NcclTransport (ZMQ PUT_BUNDLE header
    + ncclSend/ncclRecv on a 2-rank communicator per pair) and its paged-block
    extract/inject utilities, in the order its connector runs them in overlap
    mode "off" (one message per request)."""
    from kvserve_v1.compression.manager import add_sentinel  # noqa: E402
    from kvserve_v1.compression.wire import (CompressedWire, build_wire,  # noqa: E402
                                              restore_from_wire)
    from kvserve_v1.transport.nccl_transport import NcclTransport  # noqa: E402
    from kvserve_v1.utils.kv_utils import (extract_kv_from_layer_by_blocks,  # noqa: E402
                                           inject_kv_into_layer_by_blocks)
    import threading
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    pairs = world // 2
    role = "producer" if rank < pairs else "consumer"
    pair_id = rank % pairs
    raw = args.compression == "off"
    pipe = None if raw else _RefPipeline(args)
    wl = Workload(args, device, args.seed + 101 * pair_id, role)
    L = args.layers
    plain_names = [f"model.layers.{l}.self_attn.attn" for l in range(L)]
    names = add_sentinel(plain_names)
    tr = _REF_TRANSPORTS.get((role, pair_id))
    if tr is None:  # one communicator per pair for the life of the process
        tr = NcclTransport(role == "producer", "127.0.0.1", side_port(500, pair_id), local, 0)
        _REF_TRANSPORTS[(role, pair_id)] = tr
    pending: dict = {}
    sizes = []

    def wait_sent(timeout_s=120.0):
        t = threading.Thread(target=tr.wait_for_sent, daemon=True)
        t.start()
        t.join(timeout_s)
        if t.is_alive():
            raise TimeoutError("reference sends did not complete")

    def step(s):
        for r in range(wl.B):
            key = f"s{s}r{r}"
            if role == "producer":
                stacked = torch.stack([extract_kv_from_layer_by_blocks(wl.src[l], wl.src_req[r][0])
                                       for l in range(L)], dim=0)
                if raw:
                    sizes.append(int(stacked.numel() * stacked.element_size()))
                    tr.send(key, plain_names, stacked)
                    continue
                c = pipe.compress(stacked, key)
                w = build_wire(c, 512 << 20)  # the connector's default chunk bound
                sizes.append(int(w.nbytes))
                tr.send_bundle(key, names, w.meta, w.body_chunks, w.aux_tensors)
            else:
                _, payload = _poll_message(tr, pending, key, 120.0)
                if raw or isinstance(payload, torch.Tensor):
                    out = payload
                else:
                    cd = restore_from_wire(CompressedWire(payload["meta"], payload["body_chunks"],
                                                          payload["aux_tensors"]))
                    out = pipe.decompress(cd)
                for l in range(L):
                    inject_kv_into_layer_by_blocks(wl.dst[l], out[l], wl.dst_req[r][0])

    s = 0
    for _ in range(args.warmup):
        step(s)
        s += 1
    if role == "producer":
        wait_sent()
    torch.cuda.synchronize(device)
    barrier(world)
    sampler = ClockSampler(range(world)) if local == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)

    def timed(s):
        step(s)

    barrier(world)
    torch.cuda.synchronize(device)
    ev0, ev1 = _events()
    ev0.record()
    for _ in range(args.steps):
        timed(s)
        s += 1
    if role == "producer":
        wait_sent()
    ev1.record()
    torch.cuda.synchronize(device)
    ms = allreduce_max(ev0.elapsed_time(ev1), world)
    barrier(world)
    clocks = sampler.stop() if sampler else None
    err = None
    if role == "consumer":
        src = Workload(args, device, args.seed + 101 * pair_id, "producer")
        err = _ref_error(src, wl, device)
        del src
    err = first_non_none(err, world)
    tot = allreduce_sum(float(sum(sizes[-args.steps * wl.B:])), world)
    n = allreduce_sum(float(len(sizes[-args.steps * wl.B:])), world)
    cr = wl.bf16_bytes_per_request / (tot / n) if n else None
    nb = len((wl.src_req if role == "producer" else wl.dst_req)[0][0])
    cache, blocks = (wl.src[L - 1], wl.src_req[-1][0]) if role == "producer" else \
        (wl.dst[L - 1], wl.dst_req[-1][0])
    e2e = None if args.no_e2e else _ref_e2e(
        args, world, device, step, s, cache, blocks, 2 * wl.B * L * nb * 8, pairs,
        finish=wait_sent if role == "producer" else None)
    return {"ms": ms, "cr": cr, "error": err, "clocks": clocks, "pairs": pairs, "e2e": e2e,
            "pipeline": ("raw: extract_kv_from_layer_by_blocks + stack + NcclTransport.send "
                         "+ inject_kv_into_layer_by_blocks") if raw else
                        REF_PIPELINE + "; its build_wire + NcclTransport.send_bundle",
            "transport": "reference NcclTransport (ZMQ header + NCCL send/recv per pair)"}


# ------------------------------------------------------------------ main
def build_line(args, res, world):
    """The one JSON line rank 0 prints."""
    pairs = res.get("pairs", 1)
    per_pair_requests = args.steps * args.requests_per_step
    value = res["ms"] / per_pair_requests
    raw_bytes = args.layers * 2 * args.tokens * args.kv_heads * 128 * 2
    line = {
        "metric": METRIC,
        "value": round(value, 5),
        "unit": "ms/request",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(res["ms"] / args.steps, 4),
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: N(0,1) bf16 KV, 3% outlier key channels x12, shuffled 16-token "
                "blocks; Qwen2.5-7B KV shapes (random-init, no checkpoint)",
        "config": {
            "model": "Qwen2.5-7B (28 layers, 4 KV heads, head_dim 128)",
            "global_batch": args.requests_per_step * pairs,
            "seq_len": args.tokens,
            "parallelism": "1-GPU round trip" if world == 1 else f"1P1D x{pairs} pairs (TP1)",
            "compression": compression_label(args),
            "requests_per_step": args.requests_per_step,
            "kv_layout": ("HND head-major blocks (vLLM FlashInfer on B200)"
                          if args.kv_layout == "hnd" else "NHD token-major blocks"),
            "value_definition": "ms per request of one producer/consumer pair (N=1: one GPU "
                                "does both halves)",
            "l2": "inputs larger than L2 (%.1f GB of KV per step per producer)"
                  % (raw_bytes * args.requests_per_step / 1e9),
        },
        "compression_ratio": round(res["cr"], 3) if res.get("cr") else None,
        "reconstruction": res.get("error"),
        "clocks": res.get("clocks"),
        "aggregate_gbps": round(raw_bytes * args.requests_per_step * pairs * args.steps /
                                (res["ms"] * 1e6), 1),
        "pipeline": res.get("pipeline"),
        "transport": res.get("transport"),
    }
    for k in ("stage_ms_per_request", "single_request_latency_ms", "full_path"):
        if res.get(k) is not None:
            line[k] = res[k]
    if args.compression != "off":  # same config, same algorithmic bytes in both arms
        line["roofline"] = roofline(args, world, res.get("codec", args.codec), res.get("cr"),
                                    value)
    if args.impl == "reference":
        line["impl"] = "reference"
        if res.get("e2e"):
            line["e2e"] = res["e2e"]
    else:
        line["impl"] = "ours"
        line["gpu_launches"] = int(res.get("launches_job", res.get("launches_total",
                                                                  res["launches"])))
        line["engine"] = args.engine
        if res.get("e2e"):
            line["e2e"] = res["e2e"]
        if res.get("device_error"):
            line["device_error"] = res["device_error"]
    return line


def main(argv=None):
    args = parse_args(argv)
    rank, world, local = dist_info()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if args.warmup < 3:  # timed numbers need at least three untimed warm-up steps
        print(f"bench: --warmup {args.warmup} raised to 3", file=sys.stderr)
        args.warmup = 3
    init_dist(world, local)
    if args.impl == "reference":
        res = run_reference(args, rank, world, local)
    else:
        res = run_ours(args, rank, world, local)
    if "unavailable" in res:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": res["unavailable"]}), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return 0
    if args.impl == "ours" and res.get("pipeline") is None:
        res["pipeline"] = ("fused sm_100a kernels: tcgen05 Hadamard (TMA from the paged cache) "
                           "+ hybrid quantization, " + ("rANS, " if res.get("codec") == "rans"
                                                        else "") +
                           "dequantization + inverse Hadamard + paged scatter")
    if args.impl == "ours":  # every rank's own kernels, summed over the job
        total = res.get("launches_total", res["launches"])
        res["launches_job"] = allreduce_sum(float(total), world) if world > 1 else total
    line = build_line(args, res, world)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        barrier(world)
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
