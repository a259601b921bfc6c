#!/usr/bin/env python
"""KV-handoff benchmark: per-request prefill->decode KV transfer time.

Metric: "PD KV-transfer ms/request & p50 TTFT (Qwen2.5-7B,
8K prompt); compression ratio".  Config: Qwen2.5-7B KV shapes (28 layers,
4 KV heads, head_dim 128), 8192-token prompts, default compression mode,
synthetic N(0,1) KV with 3% outlier key channels x12 stored in a paged cache
(16-token blocks) at shuffled block ids.

One step hands off ``--requests-per-step`` requests:
* N = 1: round trip on one GPU -- fused quantize of every (layer, request)
  item from the paged cache, rANS encode, rANS decode, fused dequantize +
  inverse transform + scatter into a second paged cache;
* N >= 2 (torchrun, one rank per GPU): ranks [0, N/2) are producers, rank
  r + N/2 is r's consumer.  The producer's encoder writes the stream
  straight into the consumer's receive slot over NVLink and publishes a
  ready flag; the consumer waits (bounded) on the flag, decodes and scatters
  into its paged cache, then returns a credit flag to the producer.

``value`` is the job-wide device time divided by the requests handed off
by the whole job (ms/request, lower is better): each rank times its stream
with CUDA events between barriers, the maximum over ranks is used.

``--impl reference`` runs the unmodified reference package from
``baseline/_ref`` through its public ``KVCompressionAdapter`` on the same
workload.  Its default mode needs nvCOMP, CuPy and fast_hadamard_transform,
which are not installed, so the arm runs its quantizer-only custom pipeline
(the degraded mode of its own tests) and, for N >= 2, its NcclTransport.
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

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "PD KV-transfer ms/request & p50 TTFT (Qwen2.5-7B, 8K prompt); compression ratio"
MODEL = "Qwen2.5-7B-Instruct"


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
    ap.add_argument("--codec", default="rans", choices=["rans", "bitpack", "none"])
    ap.add_argument("--engine", default="tcgen05", choices=["tcgen05", "simt"])
    ap.add_argument("--compression", default="default", choices=["default", "off"],
                    help="off: raw KV blocks (no transform, quantization or codec)")
    ap.add_argument("--hybrid-ratio", type=float, default=None,
                    help="override the default mode's hybrid_ratio")
    ap.add_argument("--no-e2e", action="store_true")
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
        self.window = None

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

    def mark(self, t0, t1):
        self.window = (t0, t1)

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
class Workload:
    """Source and destination paged caches for one rank."""

    def __init__(self, args, device, seed, role="both"):
        from kvserve_hpdps_b200.models.synthetic import outlier_channels
        L, H, bs, T, B = args.layers, args.kv_heads, args.block_size, args.tokens, args.requests_per_step
        nb = (T + bs - 1) // bs
        self.nblocks = B * nb + 7
        self.L, self.H, self.bs, self.T, self.B, self.nb = L, H, bs, T, B, nb
        g = torch.Generator(device="cpu").manual_seed(seed)
        perm_src = torch.randperm(self.nblocks, generator=g).tolist()
        perm_dst = torch.randperm(self.nblocks, generator=g).tolist()
        self.src_req = [(perm_src[i * nb:(i + 1) * nb], T) for i in range(B)]
        self.dst_req = [(perm_dst[i * nb:(i + 1) * nb], T) for i in range(B)]
        shape = (L, 2, self.nblocks, bs, H, 128)
        self.src = self.dst = None
        if role in ("both", "producer"):
            self.src = torch.empty(shape, dtype=torch.bfloat16, device=device)
            gd = torch.Generator(device=device).manual_seed(seed + 17)
            for l in range(L):  # fill layer by layer to bound temporaries
                self.src[l].normal_(generator=gd)
            m = outlier_channels(H, 128, fraction=0.03, seed=seed + 3).to(device)
            scale = torch.where(m, 12.0, 1.0).to(torch.bfloat16)
            for l in range(L):
                self.src[l, 0].view(-1, H, 128).mul_(scale)
        if role in ("both", "consumer"):
            self.dst = torch.zeros(shape, dtype=torch.bfloat16, device=device)

    @property
    def bf16_bytes_per_request(self) -> int:
        return self.L * 2 * self.T * self.H * 128 * 2


def quant_config(args):
    from kvserve_hpdps_b200.compression.config import get_default_compression_config
    cfg = get_default_compression_config()
    cfg["quantizer_config"]["model_name"] = MODEL
    if getattr(args, "hybrid_ratio", None) is not None:
        cfg["quantizer_config"]["hybrid_ratio"] = float(args.hybrid_ratio)
    if args.codec == "bitpack":
        cfg["codec_config"] = {"codec_type": "bitpack"}
    elif args.codec == "none":
        cfg["codec_config"] = {"codec_type": "none"}
    return cfg


# ------------------------------------------------------------------ ours
def _roles(world, rank):
    pairs = max(1, world // 2)
    if world == 1:
        return "both", pairs
    if world % 2:
        raise SystemExit("--gpus must be 1 or even")
    return ("producer" if rank < pairs else "consumer"), pairs


def _timed(step, args, world, local, device, s0):
    """Warm-up, then ``args.steps`` steps between barriers and device
    synchronisations, timed with CUDA events; returns (max ms over ranks,
    clocks, next step index, device error)."""
    from kvserve_hpdps_b200.ops import kernels as K
    s = s0
    for _ in range(args.warmup):
        step(s)
        s += 1
    torch.cuda.synchronize(device)
    err = K.read_device_error(device)
    if err:
        raise RuntimeError(f"device error {err} during warmup ({K.ERR_NAMES.get(err)})")
    sampler = ClockSampler(range(world)) if local == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        step(s)
        s += 1
    ev1.record()
    torch.cuda.synchronize(device)
    barrier(world)
    ms = ev0.elapsed_time(ev1)
    err = K.read_device_error(device)
    clocks = sampler.stop() if sampler else None
    return allreduce_max(ms, world), clocks, s, int(allreduce_max(float(err), world))


def run_ours_raw(args, rank, world, local):
    """Compression off: raw KV blocks.  N = 1: one gather launch of every
    (layer, request) item from the paged cache into a flat buffer and one
    scatter launch into the second cache.  N >= 2: the producer's gather
    stores straight into the consumer's receive slot over NVLink and
    publishes a ready flag; the consumer waits (bounded) on it and scatters
    into its cache, then returns a credit flag."""
    from kvserve_hpdps_b200.ops import kernels as K
    device = torch.device("cuda", local)
    role, pairs = _roles(world, rank)
    pair_id = rank % pairs
    wl = Workload(args, device, args.seed + 101 * pair_id, role)
    L = args.layers
    layers_src = [wl.src[l] for l in range(L)] if wl.src is not None else None
    layers_dst = [wl.dst[l] for l in range(L)] if wl.dst is not None else None
    src_raw = K.RawItems(layers_src, [(l, b) for b, _ in wl.src_req for l in range(L)]) \
        if layers_src else None
    dst_raw = K.RawItems(layers_dst, [(l, b) for b, _ in wl.dst_req for l in range(L)]) \
        if layers_dst else None
    nbytes = (src_raw or dst_raw).flat_bytes
    slot_bytes = ((nbytes + 255) // 256) * 256
    if world == 1:
        flat = torch.empty(nbytes, dtype=torch.uint8, device=device)

        def step(s):
            K.paged_raw(src_raw, flat.data_ptr(), True)
            K.paged_raw(dst_raw, flat.data_ptr(), False)
        launches = 2
        transport = "local"
    else:
        import torch.distributed as dist
        from kvserve_hpdps_b200.parallel.p2p import DeviceRegion, PeerMapping
        peer = rank + pairs if role == "producer" else rank - pairs
        region = DeviceRegion(local, 2 * slot_bytes + 4096) if role == "consumer" else \
            DeviceRegion(local, 4096)
        handles = [None] * world
        dist.all_gather_object(handles, (region.ipc_handle(), region.nbytes, local))
        ph, pn, _ = handles[peer]
        peer_map = PeerMapping(local, ph, pn)

        def step(s):
            slot = s % 2
            if role == "producer":
                if s >= 2:
                    K.wait_flag(region.ptr + 256 * slot, s - 1, device, timeout_s=20.0)
                K.paged_raw(src_raw, peer_map.ptr + slot * slot_bytes, True,
                            flag_ptr=peer_map.ptr + 2 * slot_bytes + 256 * slot, flag_value=s + 1)
            else:
                K.wait_flag(region.ptr + 2 * slot_bytes + 256 * slot, s + 1, device,
                            timeout_s=20.0)
                K.paged_raw(dst_raw, region.ptr + slot * slot_bytes, False)
                K.set_flag(peer_map.ptr + 256 * slot, s + 1, device)
        launches = 2 if role == "producer" else 3
        transport = "nvlink-p2p (one gather launch stores raw blocks into the consumer's slot)"

    ms, clocks, _, err = _timed(step, args, world, local, device, 0)
    error = None
    if role in ("both", "consumer"):
        ref = wl if wl.src is not None else Workload(args, device, args.seed + 101 * pair_id,
                                                     "producer")
        idx_s = torch.tensor(ref.src_req[0][0], device=device)
        idx_d = torch.tensor(wl.dst_req[0][0], device=device)
        error = {"exact": bool(torch.equal(ref.src[:, :, idx_s], wl.dst[:, :, idx_d]))}
        del ref
    if world > 1:
        import torch.distributed as dist
        gathered = [None] * world
        dist.all_gather_object(gathered, error)
        error = next((g for g in gathered if g is not None), None)
        barrier(world)
        peer_map.close()
        barrier(world)
        region.close()
    return {"ms": ms, "cr": 1.0, "error": error, "transport": transport,
            "launches": launches * args.steps, "clocks": clocks, "e2e": None,
            "device_error": err, "pairs": pairs, "role": role}


def run_ours(args, rank, world, local):
    if getattr(args, "compression", "default") == "off":
        return run_ours_raw(args, rank, world, local)
    from kvserve_hpdps_b200.compression.fused_manager import FusedCompressionManager
    from kvserve_hpdps_b200.ops import kernels as K
    device = torch.device("cuda", local)
    cfg = quant_config(args)
    engine = 1 if args.engine == "simt" else 0
    mgr = FusedCompressionManager(args.kv_heads, 128, cfg["quantizer_config"], cfg["codec_config"],
                                  engine=engine)
    pairs = max(1, world // 2)
    if world == 1:
        role = "both"
    else:
        if world % 2:
            raise SystemExit("--gpus must be 1 or even")
        role = "producer" if rank < pairs else "consumer"
    pair_id = rank % pairs
    wl = Workload(args, device, args.seed + 101 * pair_id, role)
    L = args.layers
    plans = [mgr.plan(l) for l in range(L)]
    src_slots = K.LayerSlots([wl.src[l] for l in range(L)], plans) if wl.src is not None else None
    dst_slots = K.LayerSlots([wl.dst[l] for l in range(L)], plans) if wl.dst is not None else None
    any_slots = src_slots or dst_slots
    src_items = K.WorkItems(any_slots, [(l, b, n) for l in range(L) for b, n in wl.src_req])
    dst_items = K.WorkItems(any_slots if dst_slots is None else dst_slots,
                            [(l, b, n) for l in range(L) for b, n in wl.dst_req])
    code_bytes = src_items.code_bytes
    meta_bytes = src_items.meta_bytes
    codes = torch.empty(code_bytes, dtype=torch.uint8, device=device)
    meta = torch.empty(meta_bytes, dtype=torch.uint8, device=device)
    cap = K.rans_max_bytes(code_bytes) if mgr.stream_codec == "rans" else code_bytes
    slot_bytes = ((cap + meta_bytes + 255) // 256) * 256
    dec_codes = torch.empty(code_bytes, dtype=torch.uint8, device=device)
    launches_per_step = 0
    use_rans = mgr.stream_codec == "rans"

    if world == 1:
        stream_buf = torch.empty(cap, dtype=torch.uint8, device=device)

        def step(s):
            K.quantize(src_slots, src_items, codes, meta, engine=engine)
            if use_rans:
                K.rans_encode_ptr(codes.data_ptr(), code_bytes, stream_buf.data_ptr(), device)
                K.rans_decode_ptr(stream_buf.data_ptr(), code_bytes, dec_codes.data_ptr(), device,
                                  stream_bytes=cap)
                K.dequantize(dec_codes, meta, dst_slots, dst_items, engine=engine)
            else:
                K.dequantize(codes, meta, dst_slots, dst_items, engine=engine)
        launches_per_step = 3 + (5 if use_rans else 1)
        transport = "local"
    else:
        import torch.distributed as dist
        from kvserve_hpdps_b200.parallel.p2p import DeviceRegion, PeerMapping
        peer = rank + pairs if role == "producer" else rank - pairs
        # consumer: 2 receive slots (stream + meta) + ready flags; producer: credit flags
        region = DeviceRegion(local, 2 * slot_bytes + 4096) if role == "consumer" else \
            DeviceRegion(local, 4096)
        handles = [None] * world
        dist.all_gather_object(handles, (region.ipc_handle(), region.nbytes, local))
        ph, pn, pdev = handles[peer]
        peer_map = PeerMapping(local, ph, pn)
        flags_off = 2 * slot_bytes if role == "consumer" else 0

        def step(s):
            slot = s % 2
            if role == "producer":
                if s >= 2:  # receive slot reused: wait for the consumer's credit
                    K.wait_flag(region.ptr + 256 * slot, s - 1, device, timeout_s=20.0)
                K.quantize(src_slots, src_items, codes, meta, engine=engine)
                dst = peer_map.ptr + slot * slot_bytes
                K.copy_bytes(meta.data_ptr(), dst + cap, meta_bytes, device)
                flag = peer_map.ptr + 2 * slot_bytes + 256 * slot
                if use_rans:
                    K.rans_encode_ptr(codes.data_ptr(), code_bytes, dst, device, flag_ptr=flag,
                                      flag_value=s + 1)
                else:
                    K.copy_bytes(codes.data_ptr(), dst, code_bytes, device, flag_ptr=flag,
                                 flag_value=s + 1)
            else:
                base = region.ptr + slot * slot_bytes
                K.wait_flag(region.ptr + flags_off + 256 * slot, s + 1, device, timeout_s=20.0)
                K.copy_bytes(base + cap, meta.data_ptr(), meta_bytes, device)
                if use_rans:
                    K.rans_decode_ptr(base, code_bytes, dec_codes.data_ptr(), device,
                                      stream_bytes=cap)
                    K.dequantize(dec_codes, meta, dst_slots, dst_items, engine=engine)
                else:
                    K.copy_bytes(base, dec_codes.data_ptr(), code_bytes, device)
                    K.dequantize(dec_codes, meta, dst_slots, dst_items, engine=engine)
                K.set_flag(peer_map.ptr + 256 * slot, s + 1, device)
        launches_per_step = (1 + 3 + 1 + 3) if role == "producer" else (1 + 1 + 2 + 1)
        transport = "nvlink-p2p (producer kernels store into the consumer's IPC receive slots)"

    # ---------------- warmup + correctness/CR sample (untimed)
    s_global = 0
    for _ in range(args.warmup):
        step(s_global)
        s_global += 1
    torch.cuda.synchronize(device)
    err = K.read_device_error(device)
    if err:
        raise RuntimeError(f"device error {err} during warmup ({K.ERR_NAMES.get(err)})")
    stats = {}
    if role in ("both", "producer"):
        if use_rans:
            probe_buf = torch.empty(cap, dtype=torch.uint8, device=device)
            sz = K.rans_encode(codes, out=probe_buf, trim=True).numel()
        else:
            sz = code_bytes
        stats["stream_bytes"] = sz + meta_bytes
    if role in ("both", "consumer"):
        # a pair's consumer regenerates its producer's (deterministic) source
        ref_wl = wl if wl.src is not None else Workload(args, device, args.seed + 101 * pair_id,
                                                          "producer")
        idx_s = torch.tensor(ref_wl.src_req[0][0], device=device)
        idx_d = torch.tensor(wl.dst_req[0][0], device=device)
        stats["error"] = K.kv_error(ref_wl.src[:, :, idx_s], wl.dst[:, :, idx_d])
        if ref_wl is not wl:
            del ref_wl

    # ---------------- timed region
    sampler = ClockSampler(range(world)) if local == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        step(s_global)
        s_global += 1
    ev1.record()
    torch.cuda.synchronize(device)
    barrier(world)
    ms = ev0.elapsed_time(ev1)
    err = K.read_device_error(device)
    clocks = sampler.stop() if sampler else None
    ms_max = allreduce_max(ms, world)
    err_any = allreduce_max(float(err), world)

    # ---------------- end-to-end through the public API
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e_ours(args, mgr, wl, role, world, rank, pairs, device)

    # aggregate compression stats; reconstruction error from a consumer rank
    if world > 1:
        import torch.distributed as dist
        gathered = [None] * world
        dist.all_gather_object(gathered, stats.get("error"))
        stats["error"] = next((g for g in gathered if g is not None), None)
        barrier(world)  # unmap the peer slot before its owner frees it
        peer_map.close()
        barrier(world)
        region.close()
    stream_bytes = allreduce_sum(float(stats.get("stream_bytes", 0)), world)
    n_prod = pairs if world > 1 else 1
    orig = wl.bf16_bytes_per_request * wl.B * n_prod
    cr = orig / stream_bytes if stream_bytes else None
    out = {
        "ms": ms_max, "cr": cr, "error": stats.get("error"), "transport": transport,
        "launches": launches_per_step * args.steps, "clocks": clocks, "e2e": e2e,
        "device_error": int(err_any), "pairs": n_prod, "role": role,
    }
    return out


def run_e2e_ours(args, mgr, wl, role, world, rank, pairs, device):
    """End to end through the public manager API.

    Every step copies the step's request descriptors (block tables, token
    counts) from pinned host memory to the device, compresses the requests'
    KV into one wire message (``compress_paged_requests``, which reads the
    stream size back to the host), and decompresses it into the consumer's
    paged cache (``decompress_paged_requests``), then reads the device error
    word back.  With N >= 2 the message travels by NCCL send/recv between the
    pair (public wire envelope path)."""
    from kvserve_hpdps_b200.ops import kernels as K
    L = wl.L
    h2d = d2h = 0
    steps = max(2, min(args.steps, 10))

    def one():
        nonlocal h2d, d2h
        if role == "both":
            cd = mgr.compress_paged_requests([wl.src[l] for l in range(L)], list(range(L)),
                                             wl.src_req, trim=False)
            mgr.decompress_paged_requests(cd, [wl.dst[l] for l in range(L)], wl.dst_req)
            return
        raise NotImplementedError

    if world > 1:
        return run_e2e_pairs(args, mgr, wl, role, world, rank, pairs, device)
    for _ in range(2):
        one()
    torch.cuda.synchronize(device)
    K.reset_transfer_counters()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(steps):
        one()
        K.read_device_error(device)
    ev1.record()
    torch.cuda.synchronize(device)
    ms = ev0.elapsed_time(ev1)
    c = K.transfer_counters()
    return {"value": ms / (steps * wl.B), "unit": "ms/request",
            "h2d_bytes_per_step": c["h2d"] // steps, "d2h_bytes_per_step": c["d2h"] // steps + 4,
            "steps": steps}


def side_port(offset, pair_id):
    return int(os.environ.get("MASTER_PORT", "29500")) + offset + pair_id


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
        time.sleep(2e-5)
    return pending[key].pop(0)


def run_e2e_pairs(args, mgr, wl, role, world, rank, pairs, device):
    """End to end through the public API on producer/consumer pairs: the
    producer compresses the step's requests into one grouped message
    (``compress_paged_requests``), builds the wire envelope and hands it to
    the NVLink ring transport (``P2PTransport.send_bundle``: ZMQ header,
    device stores into the consumer's receive ring); the consumer drains the
    transport, waits on the ring flag, restores the envelope and decodes into
    its paged cache (``decompress_paged_requests``), then reads the device
    error word back.  Block tables go host -> device every step."""
    from kvserve_hpdps_b200.compression.manager import add_sentinel
    from kvserve_hpdps_b200.compression.wire import CompressedWire, build_wire, restore_from_wire
    from kvserve_hpdps_b200.ops import kernels as K
    from kvserve_hpdps_b200.parallel.p2p_transport import P2PTransport
    L = wl.L
    pair_id = rank % pairs
    tr = P2PTransport(role == "producer", "127.0.0.1", side_port(600, pair_id), device.index,
                      0, ring_bytes=int(os.environ.get("KVSERVE_RING_BYTES", str(2 << 30))))
    names = add_sentinel([f"model.layers.{l}.self_attn.attn" for l in range(L)])
    pending: dict = {}
    steps = max(2, min(args.steps, 10))

    def one(s):
        if role == "producer":
            cd = mgr.compress_paged_requests([wl.src[l] for l in range(L)], list(range(L)),
                                             wl.src_req, member_tids=[f"{s}:{r}" for r in range(wl.B)],
                                             trim=False)
            w = build_wire(cd)
            tr.send_bundle(f"s{s}", names, w.meta, w.body_chunks, w.aux_tensors)
        else:
            _, payload = _poll_message(tr, pending, f"s{s}", 60.0)
            tr.prepare(payload, device)
            cd = restore_from_wire(CompressedWire(payload["meta"], payload["body_chunks"],
                                                  payload["aux_tensors"]))
            mgr.decompress_paged_requests(cd, [wl.dst[l] for l in range(L)], wl.dst_req)
            tr.release(payload, device)
            K.read_device_error(device)

    s = 0
    for _ in range(2):
        one(s)
        s += 1
    if role == "producer":
        tr.wait_for_sent(60.0)
    torch.cuda.synchronize(device)
    barrier(world)
    K.reset_transfer_counters()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(steps):
        one(s)
        s += 1
    if role == "producer":
        if not tr.wait_for_sent(60.0):
            raise TimeoutError("sends did not complete")
    torch.cuda.synchronize(device)
    ev1.record()
    torch.cuda.synchronize(device)
    ms = allreduce_max(ev0.elapsed_time(ev1), world)
    c = K.transfer_counters()
    h2d = allreduce_sum(float(c["h2d"]), world) / steps
    d2h = allreduce_sum(float(c["d2h"] + (4 * steps if role == "consumer" else 0)), world) / steps
    barrier(world)
    tr.close()
    return {"value": ms / (steps * wl.B * pairs), "unit": "ms/request",
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": steps,
            "path": "compress_paged_requests -> build_wire -> P2PTransport.send_bundle -> "
                    "drain_received/prepare -> restore_from_wire -> decompress_paged_requests"}


# ------------------------------------------------------------------ reference
_REF_TRANSPORTS: dict = {}


def _ref_compressed_bytes(c) -> int:
    """Compressed body bytes of the reference's CompressedKVData (a single
    tensor, or chunks above its 500 MiB chunking threshold)."""
    if getattr(c, "is_chunked", False) and c.chunks:
        return int(sum(t.numel() * t.element_size() for t in c.chunks))
    if c.compressed_tensor is not None:
        return int(c.compressed_tensor.numel() * c.compressed_tensor.element_size())
    return int(c.compressed_size)


def run_reference_pairs(args, rank, world, local):
    """Reference arm on producer/consumer pairs, through the reference's own
    public modules: its KVCompressionAdapter (quantizer pipeline), its wire
    envelope (build_wire / restore_from_wire), its NcclTransport
    (ZMQ PUT_BUNDLE header + ncclSend/ncclRecv on a 2-rank communicator per
    pair) and its paged-block extract/inject utilities, in the order its
    connector runs them in overlap mode "off"."""
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    sys.path.insert(0, ref_root)
    from kvserve_v1.compression.manager import KVCompressionAdapter, add_sentinel  # noqa: E402
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
    cfg = quant_config(args)
    spec = {"enabled": True, "pipeline": ["quantizer"],
            "quantizer_config": dict(cfg["quantizer_config"]), "min_compress_size": 0}
    raw = getattr(args, "compression", "default") == "off"
    adapter = None if raw else KVCompressionAdapter(spec, num_kv_heads=args.kv_heads,
                                                    head_size=128, model_name=MODEL)
    wl = Workload(args, device, args.seed + 101 * pair_id, role)
    L = args.layers
    plain_names = [f"model.layers.{l}.self_attn.attn" for l in range(L)]
    names = add_sentinel(plain_names)
    tr = _REF_TRANSPORTS.get((role, pair_id))
    if tr is None:  # one communicator per pair for the life of the process
        tr = NcclTransport(role == "producer", "127.0.0.1", side_port(500, pair_id), local, 0)
        _REF_TRANSPORTS[(role, pair_id)] = tr
    tag = getattr(args, "tag", "")
    pending: dict = {}
    sizes = []
    fallbacks = []  # requests its adapter returned None for (sent raw)

    def wait_sent(timeout_s=120.0):
        t = threading.Thread(target=tr.wait_for_sent, daemon=True)
        t.start()
        t.join(timeout_s)
        if t.is_alive():
            raise TimeoutError("reference sends did not complete")

    def step(s):
        for r in range(wl.B):
            key = f"{tag}s{s}r{r}"
            if role == "producer" and raw:  # the connector's path without compression
                stacked = torch.stack([extract_kv_from_layer_by_blocks(wl.src[l], wl.src_req[r][0])
                                       for l in range(L)], dim=0)
                sizes.append(int(stacked.numel() * stacked.element_size()))
                tr.send(key, plain_names, stacked)
            elif role == "producer":
                layers = [extract_kv_from_layer_by_blocks(wl.src[l], wl.src_req[r][0])
                          for l in range(L)]
                stacked = torch.stack(layers, dim=0)
                c = adapter.compress(stacked, key)
                if c is None:  # as its connector does: send the raw KV instead
                    fallbacks.append(key)
                    sizes.append(int(stacked.numel() * stacked.element_size()))
                    tr.send(key, plain_names, stacked)
                    continue
                sizes.append(_ref_compressed_bytes(c))
                w = build_wire(c, 512 << 20)  # the connector's default chunk bound
                tr.send_bundle(key, names, w.meta, w.body_chunks, w.aux_tensors)
            else:
                _, payload = _poll_message(tr, pending, key, 120.0)
                if raw or isinstance(payload, torch.Tensor):
                    out = payload
                else:
                    cd = restore_from_wire(CompressedWire(payload["meta"], payload["body_chunks"],
                                                          payload["aux_tensors"]))
                    out = adapter.decompress(cd)
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
    barrier(world)
    torch.cuda.synchronize(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        step(s)
        s += 1
    if role == "producer":
        wait_sent()
    torch.cuda.synchronize(device)
    ev1.record()
    torch.cuda.synchronize(device)
    ms = allreduce_max(ev0.elapsed_time(ev1), world)
    barrier(world)
    clocks = sampler.stop() if sampler else None
    err = None
    if role == "consumer":
        src = Workload(args, device, args.seed + 101 * pair_id, "producer")
        a = src.src[:, :, torch.tensor(src.src_req[0][0], device=device)].float()
        b = wl.dst[:, :, torch.tensor(wl.dst_req[0][0], device=device)].float()
        err = {"cosine": float(torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0)),
               "rel_mse": float(((a - b) ** 2).sum() / (a ** 2).sum())}
        del src
    import torch.distributed as dist
    gathered = [None] * world
    dist.all_gather_object(gathered, err)
    err = next((g for g in gathered if g is not None), None)
    tot = allreduce_sum(float(sum(sizes)), world)
    n = allreduce_sum(float(len(sizes)), world)
    cr = wl.bf16_bytes_per_request / (tot / n) if n else None
    nfall = allreduce_sum(float(len(fallbacks)), world)
    return {"ms": ms, "cr": cr, "error": err, "clocks": clocks, "pairs": pairs,
            "fallback_raw": int(nfall),
            "reference_path": ("raw: extract_kv_from_layer_by_blocks + stack + "
                               "NcclTransport.send (ncclSend/ncclRecv per pair) + "
                               "inject_kv_into_layer_by_blocks") if raw else
                              ("custom pipeline [quantizer] via KVCompressionAdapter + "
                               "build_wire + NcclTransport.send_bundle (ncclSend/ncclRecv per "
                               "pair)"),
            "transport": "reference NcclTransport (NCCL send/recv over NVLink)"}


def run_reference(args, rank, world, local):
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "kvserve_v1")):
        return {"unavailable": "reference not installed in baseline/_ref"}
    if world > 1:
        return run_reference_pairs(args, rank, world, local)
    sys.path.insert(0, ref_root)
    from kvserve_v1.compression.manager import KVCompressionAdapter  # noqa: E402
    from kvserve_v1.utils.kv_utils import (extract_kv_from_layer_by_blocks,  # noqa: E402
                                           inject_kv_into_layer_by_blocks)
    device = torch.device("cuda", local)
    raw = getattr(args, "compression", "default") == "off"
    path, default_err, adapter = "raw", "", None
    if not raw:
        try:
            KVCompressionAdapter("default", num_kv_heads=args.kv_heads, head_size=128,
                                 model_name=MODEL)
            path = "default"
        except Exception as e:  # noqa: BLE001
            default_err = f"{type(e).__name__}: {e}"
            path = None
        cfg = quant_config(args)
        spec = {"enabled": True, "pipeline": ["quantizer"],
                "quantizer_config": dict(cfg["quantizer_config"]), "min_compress_size": 0}
        adapter = KVCompressionAdapter(spec if path is None else "default",
                                       num_kv_heads=args.kv_heads, head_size=128,
                                       model_name=MODEL)
    wl = Workload(args, device, args.seed)
    L = args.layers
    sizes = []
    fallbacks = []

    def step(s):
        for r in range(wl.B):
            layers = [extract_kv_from_layer_by_blocks(wl.src[l], wl.src_req[r][0]) for l in range(L)]
            stacked = torch.stack(layers, dim=0)
            c = None if raw else adapter.compress(stacked, f"r{s}_{r}")
            if c is None:  # compression off, or its adapter declined: raw KV
                if not raw:
                    fallbacks.append(r)
                sizes.append(int(stacked.numel() * stacked.element_size()))
                out = stacked
            else:
                sizes.append(_ref_compressed_bytes(c))
                out = adapter.decompress(c)
            for l in range(L):
                inject_kv_into_layer_by_blocks(wl.dst[l], out[l], wl.dst_req[r][0])

    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize(device)
    sampler = ClockSampler([local])
    sampler.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for s in range(args.steps):
        step(1000 + s)
    ev1.record()
    torch.cuda.synchronize(device)
    ms = ev0.elapsed_time(ev1)
    clocks = sampler.stop()
    idx_s = torch.tensor(wl.src_req[0][0], device=device)
    idx_d = torch.tensor(wl.dst_req[0][0], device=device)
    from kvserve_hpdps_b200.compression.oracle import error_metrics
    a = wl.src[:, :, idx_s].float()
    b = wl.dst[:, :, idx_d].float()
    err = {"cosine": float(torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0)),
           "rel_mse": float(((a - b) ** 2).sum() / (a ** 2).sum())}
    del error_metrics
    cr = wl.bf16_bytes_per_request / statistics.mean(sizes)
    ref_path = ("raw: extract_kv_from_layer_by_blocks + stack + inject_kv_into_layer_by_blocks"
                if raw else "custom pipeline [quantizer] via KVCompressionAdapter (default mode "
                "unavailable: " + (default_err if path is None else "n/a") + ")")
    return {"ms": ms, "cr": cr, "error": err, "clocks": clocks, "reference_path": ref_path,
            "transport": "local", "fallback_raw": len(fallbacks)}


# ------------------------------------------------------------------ main
def hybrid_ratio(args) -> float:
    return float(quant_config(args)["quantizer_config"]["hybrid_ratio"])


def compression_label(args) -> str:
    if args.compression == "off":
        return "off (raw bf16 blocks)"
    codec = "rANS" if args.codec == "rans" else args.codec
    return f"default (Hadamard + hybrid {hybrid_ratio(args)} 12/8/6/4 + {codec})"


def main(argv=None):
    args = parse_args(argv)
    rank, world, local = dist_info()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if args.warmup < 3:  # timed numbers need at least three untimed warm-up steps
        print(f"bench: --warmup {args.warmup} raised to 3", file=sys.stderr)
        args.warmup = 3
    init_dist(world, local)
    try:
        res = run_reference(args, rank, world, local) if args.impl == "reference" else \
            run_ours(args, rank, world, local)
    finally:
        pass
    if "unavailable" in res:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": res["unavailable"]}), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return 0
    pairs = res.get("pairs", 1)
    reqs = args.steps * args.requests_per_step * pairs
    value = res["ms"] / reqs
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
            "l2": "inputs larger than L2 (%.1f GB of KV per step per producer)"
                  % (args.layers * 2 * args.tokens * args.kv_heads * 256 * args.requests_per_step / 1e9),
            "transport": res.get("transport"),
        },
        "compression_ratio": round(res["cr"], 3) if res.get("cr") else None,
        "reconstruction": res.get("error"),
        "clocks": res.get("clocks"),
    }
    if args.impl == "reference":
        line["impl"] = "reference"
        if res.get("fallback_raw"):
            line["config"]["reference_fallback_raw_requests"] = res["fallback_raw"]
        line["config"]["reference_path"] = res.get("reference_path")
        line["config"]["compression"] = (
            "off (raw bf16 blocks)" if args.compression == "off" else
            f"reference quantizer pipeline, hybrid {hybrid_ratio(args)} 12/8/6/4, u8 codes, no "
            "entropy codec (its default mode needs nvCOMP, CuPy and fast_hadamard_transform)")
    else:
        line["impl"] = "ours"
        line["gpu_launches"] = int(allreduce_sum(float(res["launches"]), world)) if world > 1 \
            else res["launches"]
        line["engine"] = args.engine
        if res.get("e2e"):
            line["e2e"] = res["e2e"]
        if res.get("device_error"):
            line["device_error"] = res["device_error"]
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        barrier(world)
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
