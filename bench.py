#!/usr/bin/env python
"""Decode-attention throughput of the talker's paged KV cache on 1..8 B200s.

One step = one 28-layer talker decode step of the attention hot path for 576 seats per GPU: per layer, the fused
K/V page append + paged decode attention (GQA 16/8, d128, bf16), contexts U[200,1200], 16-token pages in a shuffled
pool sized for 576 x 1216 tokens (engine/talker.py:72-77 with BASELINE's layout). 28 distinct per-layer pools (80 GB)
exceed the 126 MB L2, so no flush is needed between steps. The step is captured in a CUDA graph and replayed.

  value  seat-steps/s over all GPUs = seats_per_gpu * N / (max over ranks of device time per step), inputs resident
  e2e    the same metric through the public API with host buffers: every step copies its q/k/v (all layers) from
         pinned host memory and reads every layer's attention output back, double-buffered on copy streams
  roofline  algorithmic HBM bytes per launch (one layer) / average launch time, against MEASURED_PEAKS.json hbm_gbs
  cpu_baseline  the reference's CPU attention path (oracle restatement of Talker._attn_ref with the page gather and the
         append, fp32, all host threads) on a bounded sample of seats, rank 0 at N=1

--impl reference times that CPU path alone (rank 0; other ranks exit) on the same metric and config.
Multi-GPU: python -m torch.distributed.run --nproc-per-node N bench.py --gpus N (seats shard with no collective; the
process group is used only for the start barrier and the max over ranks of the timing).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "qwen3-tts-engine_b200")
for _p in (REPO, PKG, os.path.join(REPO, "tests")):     # tests/: the frame harness the c5 and admit workloads drive
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "decode-attn seat-steps/s @576 seats; achieved HBM GB/s (% peak) at 1/2/4/8 GPU"
UNIT = "seat-steps/s"
SCALE = 128 ** -0.5
PAGE, CTX_LO, CTX_HI, TOKENS_PER_SEAT = 16, 200, 1200, 1216
FALLBACK_HBM_GBS = 6650.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--seats", type=int, default=576)
    p.add_argument("--layers", type=int, default=28)
    p.add_argument("--seed", type=int, default=2)
    p.add_argument("--variant", type=int, default=5, help="decode kernel variant (q3_set_decode_variant)")
    p.add_argument("--num-splits", type=int, default=0)
    p.add_argument("--prefill-kernel", type=int, default=0, help="prefill kernel (q3_set_prefill_kernel): 0 TMA, 1 single")
    p.add_argument("--ring-frame-kernel", type=int, default=6,
                   help="one-frame ring kernel (q3_set_ring_frame_kernel): 6 rows straight into registers (default), "
                        "2 scalar heads per CTA, 1 scalar CTA per head, 0 / 3 / 4 tensor cores 4 / 2 / 1 heads per "
                        "CTA, 5 TMA pipeline")
    p.add_argument("--ring-chunk-kernel", type=int, default=1,
                   help="multi-frame ring kernel (q3_set_ring_chunk_kernel): 1 one CTA per head (default), "
                        "0 / 2 / 3 tensor cores 2 / 4 / 1 heads per CTA, 4 TMA pipeline")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--no-aux", action="store_true",
                   help="skip the short timing of configs 3 / 4, the prefill and the ring attention that a 1-GPU "
                        "config-2 run adds to its line under other_configs")
    p.add_argument("--cpu-seconds", type=float, default=12.0)
    p.add_argument("--cpu-seats", type=int, default=64)
    p.add_argument("--kernel-breakdown", action="store_true",
                   help="c5: add the per-kernel device time of one replayed frame (CUPTI via torch.profiler)")
    p.add_argument("--workload", choices=["c2", "c3", "c4", "c5", "admit", "prefill", "ring"], default="c2",
                   help="c2: the headline decode step (default); c3: 1.7B decode + chunked-prefill mix; c4: CP steps")
    return p.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def read_hbm_peak(path):
    """The measured HBM copy bandwidth (GB/s) from a peaks file: the top-level `hbm_gbs`, else the first numeric entry
    whose key names HBM (top level or one level down, e.g. {"hbm": {"gbs": ...}}); None when absent or unreadable."""
    try:
        data = json.load(open(path))
    except (OSError, ValueError):
        return None
    if not isinstance(data, dict):
        return None
    v = data.get("hbm_gbs")
    if isinstance(v, (int, float)) and v > 0:
        return float(v)
    for k, v in data.items():
        if "hbm" not in str(k).lower():
            continue
        if isinstance(v, (int, float)) and v > 0:
            return float(v)
        if isinstance(v, dict):
            for kk, vv in v.items():
                if isinstance(vv, (int, float)) and vv > 0 and "gb" in str(kk).lower():
                    return float(vv)
    return None


def hbm_peak():
    v = read_hbm_peak(os.path.join(REPO, "MEASURED_PEAKS.json"))
    return (v, "measured") if v is not None else (FALLBACK_HBM_GBS, "fallback")


def reduce_max(x, pg, device):
    """Max of a per-rank timing over all ranks (pg = torch.distributed, or None for one process)."""
    if pg is None:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def layout_for_rank(seed, rank, seats):
    """Rank r's seats: ctx U[200,1200] and a shuffled local page table (rank 0 == the config-2 layout)."""
    from q3attn import synth
    return synth.paged_layout(seed + 7919 * rank, B=seats, ctx_lo=CTX_LO, ctx_hi=CTX_HI, page=PAGE,
                              pages_per_seat=TOKENS_PER_SEAT // PAGE)


# ----------------------------------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = "clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown," \
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown," \
             "clocks_event_reasons.sw_power_cap"

    def __init__(self, device_index):
        self.proc = None
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            ident = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            ident = str(device_index)
        self.cmd = ["nvidia-smi", "-i", ident, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]

    def start(self):
        try:
            self.proc = subprocess.Popen(self.cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = []
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                rows.append(dict(sm=float(f[0]), smax=float(f[1]), power=float(f[2]), hw=f[4], hwt=f[5], swt=f[6], pcap=f[7]))
            except ValueError:
                continue
        if not rows:
            return None
        load = [r for r in rows if r["power"] > 250.0] or rows
        reasons = set()
        for r in load:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"), ("swt", "sw_thermal_slowdown"),
                              ("pcap", "sw_power_cap")):
                if r[key].lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in load), "sm_max_mhz": max(r["smax"] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows), "samples_under_load": len(load),
                "power_w_max": max(r["power"] for r in rows)}


# ----------------------------------------------------------------------------------------------------- CPU path
def cpu_sample(lay, seed, n_seats):
    """K/V of a sample of seats of the workload (one layer), fp32 on the host, plus the sampled seats' q/k/v."""
    from q3attn import synth
    pick = torch.linspace(0, lay.B - 1, n_seats).long()
    pps = lay.block_table.shape[1]
    g = synth.cpu_gen(seed + 31)
    kp = synth.randn((n_seats * pps, PAGE, 8, 128), g, 0.5)
    vp = synth.randn((n_seats * pps, PAGE, 8, 128), g, 0.5)
    bt = torch.randperm(n_seats * pps, generator=g).view(n_seats, pps).to(torch.int32)
    q = synth.randn((n_seats, 16, 128), g, 0.5)
    kn = synth.randn((n_seats, 8, 128), g, 0.5)
    vn = synth.randn((n_seats, 8, 128), g, 0.5)
    return dict(ctx=lay.ctx[pick].clone(), bt=bt, kp=kp, vp=vp, q=q, kn=kn, vn=vn, n=n_seats)


def cpu_layer(s):
    """One layer of the reference CPU path for the sampled seats: append (talker.py:72-73) + Talker._attn_ref
    (talker.py:82-88) over page-gathered K/V, fp32."""
    from oracle import attention as OA
    return OA.decode_step(s["q"], s["kn"], s["vn"], s["kp"], s["vp"], s["ctx"], s["bt"], SCALE)


def cpu_step(s, layers):
    """One step of the CPU path for the sampled seats: all `layers` layers (each one pass of the append + page gather
    + Talker._attn_ref restatement over the sample's K/V, which is larger than the host caches); returns seconds."""
    t0 = time.perf_counter()
    for _ in range(layers):
        cpu_layer(s)
    return time.perf_counter() - t0


def cpu_rate(s, layers, seconds):
    """CPU seat-steps/s over whole steps (cpu_step) repeated for at least `seconds`, after one untimed step."""
    cpu_step(s, layers)
    n, el = 0, 0.0
    while el < seconds:
        el += cpu_step(s, layers)
        n += 1
    return s["n"] * n / el, n, el


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# ----------------------------------------------------------------------------------------------------- reference arm
def run_reference(a):
    """The reference's CPU path on the host cores: each step is one whole 28-layer decode step for a bounded sample of
    the seats (cpu_step), the same unit the GPU arm's cpu_baseline times; W untimed steps, then exactly K timed ones.
    ms_per_step is the time actually measured per step (for the sampled seats); the time a step of all the config's
    seats would take on the CPU is reported separately as an extrapolation."""
    rank, _, world = dist_env()
    if rank != 0:
        return
    torch.set_num_threads(host_cores())
    lay = layout_for_rank(a.seed, 0, a.seats)
    s = cpu_sample(lay, a.seed, a.cpu_seats)
    for _ in range(max(a.warmup, 1)):
        cpu_step(s, a.layers)
    times = [cpu_step(s, a.layers) for _ in range(a.steps)]
    per_step = sum(times) / len(times)
    value = s["n"] / per_step
    sample = (f"each step: all {a.layers} layers for {s['n']} of {a.seats} seats (append + page gather + "
              f"Talker._attn_ref restated, fp32 torch CPU, {torch.get_num_threads()} threads); "
              f"seat-steps/s = sampled seats / step time")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE config 2 shapes)",
            "config": config_dict(a, world), "seats_timed_per_step": s["n"],
            "timed_s": sum(times), "step_ms_min": min(times) * 1e3, "step_ms_max": max(times) * 1e3,
            "extrapolated_ms_per_step_all_seats": per_step * 1e3 * a.seats / s["n"],
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def config_dict(a, world):
    return {"workload": "C2: 0.6B talker decode-attention step (28 layers x fused K/V append + paged decode), "
                        f"{a.seats} seats/GPU, ctx U[{CTX_LO},{CTX_HI}], page {PAGE}, shuffled page table",
            "seats_per_gpu": a.seats, "layers": a.layers, "page_size": PAGE, "heads": "16q/8kv", "head_dim": 128,
            "parallelism": f"seat-sharded x{world} (no collective)", "l2": "inputs larger than L2 (28 per-layer pools)",
            "decode_variant": a.variant}


# ----------------------------------------------------------------------------------------------------- our arm
def bench_frame(a):
    """Config 5 on one GPU: the whole frame step (28-layer talker decode with the fused q/k norm + RoPE + append +
    paged attention, codebook-0 logits and sampling, the code predictor's 16 steps x 5 layers) for 576 seats on
    random-init 0.6B weights, ctx U[200,1200], page 16, shuffled page table, greedy (top_k = 1). Device time per frame
    over CUDA-graph replays (inputs resident; the 80 GB of pools exceed L2), then end to end through Talker.step (seat
    ids from the host, the frame's codes read back every frame), then the same frame with the q/k norm + RoPE and the
    logit processing + sampling as PyTorch ops, for comparison."""
    import q3attn
    from q3attn import synth, weights
    from frame_harness import Talker
    rank, local, world = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pg = None
    if world > 1:        # seats shard with no exchange: the group only carries the start barrier and the max of times
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        pg = dist

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()

    B, page = a.seats, 16
    steps = min(a.steps, 40)                      # every frame appends one token per seat: bounded by the pool room
    seat_len = 1280                               # ctx <= 1200 plus room for 80 appended frames
    W = weights.cast(weights.random_weights(a.seed, "0.6B", max_pos=seat_len + 16), torch.bfloat16, dev)
    lay = synth.paged_layout(a.seed + 7919 * rank, B + 1, 200, 1200, page, seat_len // page)
    gen = torch.Generator(device=dev).manual_seed(a.seed * 1000 + rank)

    def build(fuse):
        t = Talker(W, B, seat_len=seat_len, buckets=[B], page=page, block_table=lay.block_table, top_k=1,
                   fuse_qk_norm_rope=fuse, fused_sampler=fuse)
        for l in range(len(W.layers)):
            t.kc[l].normal_(0.0, 0.5, generator=gen)
            t.vc[l].normal_(0.0, 0.5, generator=gen)
        t.pos[:B] = lay.ctx[:B].to(dev, torch.int64)
        t.x_in.normal_(0.0, 1.0, generator=gen)
        t.capture([B])
        t.s_seat[:B] = torch.arange(B, device=dev)
        return t

    def device_ms(t):
        pos0 = t.pos.clone()
        g = t.graphs[B]
        for _ in range(a.warmup):
            g.replay()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            g.replay()
        e1.record()
        e1.synchronize()
        barrier()
        t.pos.copy_(pos0)
        if q3attn._lib.read_status():
            raise RuntimeError("device status raised during the frame")
        return reduce_max(e0.elapsed_time(e1) / steps, pg, dev)

    t = build(True)
    clocks = ClockSampler(local)
    clocks.start()
    ms = device_ms(t)
    clk = clocks.stop()
    e2e = None
    if not a.no_e2e:
        seats = list(range(B))
        pos0 = t.pos.clone()
        for _ in range(a.warmup):
            t.step(seats).cpu()
        barrier()
        t0 = time.perf_counter()
        for _ in range(steps):
            codes = t.step(seats).cpu()
        e2e_s = reduce_max((time.perf_counter() - t0) / steps, pg, dev)
        barrier()
        t.pos.copy_(pos0)
        assert codes.shape == (B, 16)
        e2e = {"value": B * world / e2e_s, "unit": "seat-frames/s", "h2d_bytes_per_step": 8 * B,
               "d2h_bytes_per_step": 8 * 16 * B, "ms_per_frame": e2e_s * 1e3}
    breakdown = None
    if a.kernel_breakdown and rank == 0:
        breakdown = frame_kernel_breakdown(t.graphs[B], t)
    del t
    torch.cuda.empty_cache()
    t = build(False)
    ms_unfused = device_ms(t)
    del t
    torch.cuda.empty_cache()
    if pg is not None:
        pg.destroy_process_group()
    if rank != 0:
        return
    print(json.dumps({"metric": "e2e frame seat-frames/s @576 seats/GPU (0.6B random-init, greedy)", "workload": "c5",
                      "value": B * world / (ms / 1e3), "unit": "seat-frames/s", "n_gpus": world, "steps": steps,
                      "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "dtype": "bf16",
                      "scaling": "weak", "data": "synthetic (random-init weights N(0,0.02); K/V pools N(0,0.5); "
                      "ctx U[200,1200])",
                      "config": {"workload": "C5 frame: 28 talker layers + cb0 sampling + 16 CP steps x 5 layers",
                                 "seats": B, "page_size": page, "seat_len": seat_len, "sampling": "greedy (top_k=1)"},
                      "e2e": e2e, "unfused_ms_per_frame": ms_unfused,
                      "unfused": "q/k RMSNorm + RoPE and cb0 processing + top-k sampling as PyTorch ops",
                      "fusion_saves_ms_per_frame": ms_unfused - ms, "clocks": clk,
                      "kernel_breakdown": breakdown}), flush=True)


def frame_kernel_breakdown(graph, talker, top=16):
    """Per-kernel device time of two replays of a captured frame (CUPTI activity records through torch.profiler),
    as [name, us per frame, launches per frame, share]; the frame's positions are restored afterwards."""
    from torch.profiler import ProfilerActivity, profile
    pos0 = talker.pos.clone()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
    talker.pos.copy_(pos0)
    agg = {}
    for e in prof.events():
        if e.device_type.name == "CUDA":
            n, us = agg.get(e.name, (0, 0.0))
            agg[e.name] = (n + 1, us + e.device_time_total)
    total = sum(v[1] for v in agg.values())
    rows = sorted(agg.items(), key=lambda kv: -kv[1][1])[:top]
    return {"total_us_per_frame": total / 2, "launches_per_frame": sum(v[0] for v in agg.values()) // 2,
            "top": [[k[:90], round(v[1] / 2, 1), v[0] // 2, round(v[1] / total, 4)] for k, v in rows]}


def bench_admit(a):
    """Admission (engine/arrivals.py FastAdmit) on one GPU: the 0.6B talker (28 layers, random-init weights), a
    (voice, language) prefix of k = 35 shared positions and R = 42 new prompt positions per sequence, S = 1 and 8
    sequences per call: device time per replay of the admission graph (prefix copy of all layers + 27 paged-prefill
    layers + the last layer's K/V write)."""
    import q3attn
    from q3attn import weights
    from q3attn.admit import Admit
    from frame_harness import Talker
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    k, R, n_seats, seat_len = 35, 42, 64, 512
    W = weights.cast(weights.random_weights(a.seed, "0.6B", max_pos=seat_len + 16), torch.bfloat16, dev)
    T = Talker(W, n_seats, seat_len=seat_len, buckets=[8], page=16, top_k=1)
    A = Admit(T, k, R, max_slots=2, buckets=(1, 8))
    gen = torch.Generator(device=dev).manual_seed(a.seed)
    A.register_prefix(0, torch.randn(k, W.H, generator=gen, device=dev).mul_(0.5).to(torch.bfloat16))
    A.capture()
    x = torch.randn(8, R + 1, W.H, generator=gen, device=dev).mul_(0.5).to(torch.bfloat16)
    trail = torch.zeros(8, T.max_text + 1, W.H, dtype=torch.bfloat16, device=dev)
    res = {}
    for S in (1, 8):
        A.admit(list(range(S)), [0] * S, x[:S], trail[:S], [0] * S)
        g = A.graphs[S]
        for _ in range(a.warmup):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = min(a.steps, 50)
        e0.record()
        for _ in range(n):
            g.replay()
        e1.record()
        e1.synchronize()
        if q3attn._lib.read_status():
            raise RuntimeError("device status raised during admission")
        res[S] = e0.elapsed_time(e1) / n
    print(json.dumps({"metric": "admission ms per call (0.6B, k=35 shared + R=42 new positions per sequence)",
                      "workload": "admit", "value": res[8], "unit": "ms per call of 8 sequences",
                      "ms_per_call_S1": res[1], "ms_per_call_S8": res[8], "layers": len(W.layers),
                      "reference_a100": "3-4 ms GPU per admission call (engine README)"}), flush=True)


def bench_aux(a):
    """Configs 3 and 4, the prefill part of 3 and the codec ring attention (not the headline), returned as a dict:
    device time per layer on one GPU, CUDA events over graph replays, inputs resident; L2 is not flushed for c4 (its
    38 MB per-layer scratch is L2-resident by design)."""
    import q3attn
    from q3attn import synth
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peak, peak_kind = hbm_peak()
    q3attn.set_prefill_kernel(a.prefill_kernel)
    q3attn.set_ring_frame_kernel(a.ring_frame_kernel)
    q3attn.set_ring_chunk_kernel(a.ring_chunk_kernel)

    def timed(fn, n):
        s = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(s):
            fn()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                fn()
        for _ in range(a.warmup):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            g.replay()
        e1.record()
        e1.synchronize()
        if q3attn._lib.read_status():
            raise RuntimeError("device status raised")
        return e0.elapsed_time(e1) / n

    gen = torch.Generator(device=dev).manual_seed(a.seed)
    if a.workload == "prefill":
        # config 3's prefill part alone: 10 seats chunk-prefill 320-token prompts into fresh pages (a pool holding only
        # those seats: a small case for kernel profiles)
        np_, plen, pps = 10, 320, 20
        kp = torch.zeros((np_ * pps, 16, 8, 128), device=dev, dtype=torch.bfloat16)
        vp = torch.zeros_like(kp)
        bt = torch.randperm(np_ * pps, generator=torch.Generator().manual_seed(a.seed)).view(np_, pps).to(dev, torch.int32)
        T_ = np_ * plen
        qp = torch.randn((T_, 16, 128), generator=gen, device=dev, dtype=torch.bfloat16)
        kpn = torch.randn((T_, 8, 128), generator=gen, device=dev, dtype=torch.bfloat16)
        vpn = torch.randn((T_, 8, 128), generator=gen, device=dev, dtype=torch.bfloat16)
        cu = torch.arange(np_ + 1, dtype=torch.int32, device=dev) * plen
        zeros = torch.zeros(np_, dtype=torch.int32, device=dev)
        sid = torch.arange(np_, dtype=torch.int32, device=dev)

        def pre():
            q3attn.prefill_paged(qp, kpn, vpn, kp, vp, cu, cu, plen, zeros, sid, bt, SCALE, True, True)
        t_pre = timed(pre, a.steps)
        flops = 4 * 128 * 16 * np_ * (plen * (plen + 1) // 2)
        return {"metric": "chunked prefill 10 x 320 tokens into fresh pages (C3 prefill part)",
                "workload": "prefill", "value": t_pre * 1e3, "unit": "us", "tflops": flops / t_pre / 1e9,
                "flops": flops}
    if a.workload == "ring":
        # the codec decoder's windowed ring attention, one layer per launch: 256 streams, an 88-slot ring, 72-frame
        # window, fp16; heads x head_dim 16 x 64 assumed (the codec's config is not part of the checkout)
        Bs, H, hd, L, R = 256, 16, 64, 8, 88
        K = torch.randn((Bs + 1, R, L, H, hd), generator=gen, device=dev).to(torch.float16)
        V = torch.randn((Bs + 1, R, L, H, hd), generator=gen, device=dev).to(torch.float16)
        rows = torch.arange(Bs, device=dev)
        pos = torch.randint(100, 10000, (Bs,), generator=gen, device=dev)
        res = {}
        for n in (1, 4):
            q = torch.randn((Bs, n, H, hd), generator=gen, device=dev).to(torch.float16)

            def layer_calls():
                for li in range(L):
                    q3attn.ring_window_attn(q, q, q, K[:, :, li], V[:, :, li], rows, pos, 71, hd ** -0.5, False)
            ms = timed(layer_calls, a.steps)
            # bytes a layer must move: the ring rows some query of the chunk sees (min(pos, past) slots), K and V,
            # plus the chunk's q, k, v rows read and its output rows written
            vis = int(torch.clamp(pos, max=71).sum())
            byt = (2 * vis + Bs * 4 * n) * H * hd * 2
            res[n] = {"us_per_layer": ms * 1e3 / L, "gbs": byt * L / ms / 1e6}
        return {"metric": "codec decoder ring attention us per layer @256 streams (fp16, 16 x 64 heads)",
                "workload": "ring", "value": res[1]["us_per_layer"], "unit": "us per layer (1-frame chunk)",
                "chunk1": res[1], "chunk4": res[4], "layers_per_call": L,
                "reference_a100": "whole decoder call 14.1 / 44.5 ms at 256 streams x 1 / 4 frames"}
    if a.workload == "c4":
        B, L = a.seats, 5
        K = torch.randn((L, B, 8, 16, 128), generator=gen, device=dev, dtype=torch.bfloat16)
        V = torch.randn((L, B, 8, 16, 128), generator=gen, device=dev, dtype=torch.bfloat16)
        q = torch.randn((16, L, B, 16, 128), generator=gen, device=dev, dtype=torch.bfloat16)
        kv = torch.randn((2, 16, L, B, 8, 128), generator=gen, device=dev, dtype=torch.bfloat16)

        def frame():   # slot 0 then the 15 steps (n_live 1..16), 5 layers each: one launch per (step, layer)
            for p in range(16):
                for l in range(L):
                    q3attn.cp_step(q[p, l], kv[0, p, l], kv[1, p, l], K[l], V[l], p, SCALE)
        ms = timed(frame, a.steps)
        launches = 16 * L
        byt = sum(B * (4096 * (p + 1) + 12288) for p in range(16)) * L
        return {"metric": "code-predictor attention us per (step, layer) @576 seats", "workload": "c4",
                "value": ms * 1e3 / launches, "unit": "us", "frame_ms": ms, "launches_per_frame": launches,
                "bytes_per_frame": byt, "achieved_gbs": byt / ms / 1e6, "bound": "latency / L2 (not HBM)",
                "peak_hbm_gbs": peak}
    # c3: 470 decoding seats (ctx U[100,1500]) + 10 seats prefilling 320-token chunks into fresh pages, per layer
    lay, pseats, plen = synth.c3_layout(a.seed)
    nd = 470
    seq = lay.ctx[:nd].to(dev)
    bt = lay.block_table.to(dev)
    kp = torch.randn((lay.num_pages, 16, 8, 128), generator=gen, device=dev, dtype=torch.bfloat16)
    vp = torch.randn((lay.num_pages, 16, 8, 128), generator=gen, device=dev, dtype=torch.bfloat16)
    qd = torch.randn((nd, 16, 128), generator=gen, device=dev, dtype=torch.bfloat16)
    kd = torch.randn((nd, 8, 128), generator=gen, device=dev, dtype=torch.bfloat16)
    vd = torch.randn((nd, 8, 128), generator=gen, device=dev, dtype=torch.bfloat16)
    np_ = len(pseats)
    T = np_ * plen
    qp = torch.randn((T, 16, 128), generator=gen, device=dev, dtype=torch.bfloat16)
    kpn = torch.randn((T, 8, 128), generator=gen, device=dev, dtype=torch.bfloat16)
    vpn = torch.randn((T, 8, 128), generator=gen, device=dev, dtype=torch.bfloat16)
    cu = torch.arange(np_ + 1, dtype=torch.int32, device=dev) * plen
    zeros = torch.zeros(np_, dtype=torch.int32, device=dev)
    sid = torch.tensor(pseats, dtype=torch.int32, device=dev)
    btd = bt[:nd].contiguous()

    def dec():
        q3attn.paged_decode_append(qd, kd, vd, kp, vp, seq, btd, SCALE, 0)

    def pre():
        q3attn.prefill_paged(qp, kpn, vpn, kp, vp, cu, cu, plen, zeros, sid, bt, SCALE, True, True)

    def both():
        dec()
        pre()
    t_dec, t_pre, t_both = timed(dec, a.steps), timed(pre, a.steps), timed(both, a.steps)
    flops = 4 * 128 * 16 * np_ * (plen * (plen + 1) // 2)
    byt = synth.decode_bytes(lay.ctx[:nd] + 1)
    return {"metric": "1.7B talker layer: decode (470 seats) + chunked prefill (10 x 320)", "workload": "c3",
            "value": t_both * 1e3, "unit": "us per layer", "decode_us": t_dec * 1e3,
            "decode_gbs": byt / t_dec / 1e6, "decode_frac_of_hbm": byt / t_dec / 1e6 / peak,
            "prefill_us": t_pre * 1e3, "prefill_tflops": flops / t_pre / 1e9, "prefill_flops": flops,
            "peak_hbm_gbs": peak, "peak_source": peak_kind}


def main():
    a = parse()
    if a.workload == "c5" and a.impl == "ours":
        return bench_frame(a)
    if a.workload == "admit" and a.impl == "ours":
        return bench_admit(a)
    if a.workload != "c2" and a.impl == "ours":
        print(json.dumps(bench_aux(a)), flush=True)
        return
    if a.impl == "reference":
        return run_reference(a)
    import q3attn
    from q3attn import synth

    rank, local, world = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
        pg = dist
    q3attn.set_decode_variant(a.variant)

    L, B = a.layers, a.seats
    lay = layout_for_rank(a.seed, rank, B)
    seq = lay.ctx.to(dev)
    bt = lay.block_table.to(dev)
    gen = torch.Generator(device=dev).manual_seed(a.seed * 1000 + rank)
    shp = (lay.num_pages, PAGE, 8, 128)
    kp = [torch.randn(shp, generator=gen, device=dev, dtype=torch.bfloat16).mul_(0.5) for _ in range(L)]
    vp = [torch.randn(shp, generator=gen, device=dev, dtype=torch.bfloat16).mul_(0.5) for _ in range(L)]

    def inputs():
        return (torch.randn((L, B, 16, 128), generator=gen, device=dev, dtype=torch.bfloat16).mul_(0.5),
                torch.randn((L, B, 8, 128), generator=gen, device=dev, dtype=torch.bfloat16).mul_(0.5),
                torch.randn((L, B, 8, 128), generator=gen, device=dev, dtype=torch.bfloat16).mul_(0.5))

    def step(qkv):
        q, k, v = qkv
        return [q3attn.paged_decode_append(q[l], k[l], v[l], kp[l], vp[l], seq, bt, SCALE, a.num_splits) for l in range(L)]

    sets = [inputs(), inputs()] if not a.no_e2e else [inputs()]
    cap = torch.cuda.Stream(device=dev)
    graphs, outs = [], []
    with torch.cuda.stream(cap):
        for s in sets:
            step(s)
        torch.cuda.synchronize()
        for s in sets:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                o = step(s)
            graphs.append(g)
            outs.append(o)
    torch.cuda.synchronize()
    if q3attn._lib.read_status():
        raise RuntimeError("device status raised during warm-up")

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        return reduce_max(x, pg, dev)

    # ---------------- device-resident timing
    for _ in range(a.warmup):
        graphs[0].replay()
    clocks = ClockSampler(local)
    barrier()
    clocks.start()
    barrier()
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(a.steps):
        graphs[0].replay()
    e1.record(st)
    e1.synchronize()
    barrier()
    clk = clocks.stop()
    ms_total = max_over_ranks(e0.elapsed_time(e1))
    ms_step = ms_total / a.steps
    value = B * world / (ms_step / 1e3)
    if q3attn._lib.read_status():
        raise RuntimeError("device status raised during the timed region")

    # ---------------- roofline of the decode kernel (one launch == one layer)
    bytes_launch = synth.decode_bytes(lay.ctx + 1, append=True)
    launch_s = ms_step / 1e3 / L
    achieved = bytes_launch / launch_s / 1e9
    peak, peak_kind = hbm_peak()
    traffic = None
    tpath = os.path.join(REPO, "profiles", "decode_traffic_ws.json" if a.variant == 5 else "decode_traffic.json")
    if os.path.exists(tpath):
        try:
            t = json.load(open(tpath))
            traffic = t.get("dram_bytes_per_launch_scaled_to_bench") or t.get("dram_bytes_per_launch")
        except Exception:
            traffic = None
    roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "traffic": traffic, "peak_source": peak_kind, "bytes_per_launch": bytes_launch, "launch_us": launch_s * 1e6,
            "kernel": ("q3::paged_decode_ws_kernel (fused append, producer warps)" if a.variant == 5
                       else "q3::paged_decode_kernel (fused append)"),
            "resident_ctas_per_sm": int(q3attn._lib.load().q3_paged_decode_resident_ctas(a.variant))}

    # ---------------- end to end through the public API with host buffers
    e2e = None
    if not a.no_e2e:
        hq = [sets[0][i].cpu().pin_memory() for i in range(3)]
        hout = torch.empty((L, B, 16, 128), dtype=torch.bfloat16).pin_memory()
        h2d_s, d2h_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        ev_in = [torch.cuda.Event(), torch.cuda.Event()]
        ev_done = [torch.cuda.Event(), torch.cuda.Event()]
        ev_out = [torch.cuda.Event(), torch.cuda.Event()]

        def h2d(j):
            with torch.cuda.stream(h2d_s):
                for i in range(3):
                    sets[j][i].copy_(hq[i], non_blocking=True)
                ev_in[j].record(h2d_s)

        def run_e2e(n):
            h2d_s.wait_stream(st)                 # nothing of an earlier run may still read the input sets
            d2h_s.wait_stream(st)
            for j in range(2):
                ev_done[j].record(st)
                ev_out[j].record(st)
            h2d(0)
            for i in range(n):
                j = i % 2
                st.wait_event(ev_in[j])
                st.wait_event(ev_out[j])          # D2H of the step that last used this output set has finished
                graphs[j].replay()
                ev_done[j].record(st)
                if i + 1 < n:
                    h2d_s.wait_event(ev_done[1 - j])   # the previous step that read set 1-j has finished
                    h2d(1 - j)
                with torch.cuda.stream(d2h_s):
                    d2h_s.wait_event(ev_done[j])
                    for l in range(L):
                        hout[l].copy_(outs[j][l], non_blocking=True)
                    ev_out[j].record(d2h_s)
            st.wait_stream(d2h_s)
            st.wait_stream(h2d_s)

        run_e2e(max(a.warmup, 2))
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(st)
        run_e2e(a.steps)
        f1.record(st)
        f1.synchronize()
        barrier()
        e2e_ms = max_over_ranks(f0.elapsed_time(f1)) / a.steps
        elem = 2
        e2e = {"value": B * world / (e2e_ms / 1e3), "unit": UNIT, "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": int(sum(t.numel() for t in hq) * elem),
               "d2h_bytes_per_step": int(hout.numel() * elem),
               "how": "pinned host q/k/v of all layers copied in and every layer's output copied out each step, "
                      "double-buffered on two copy streams around the captured step"}
        # the copied-back outputs must equal the device-resident ones
        torch.cuda.synchronize()
        if not torch.equal(hout.view(torch.int16), torch.stack(outs[(a.steps - 1) % 2]).cpu().view(torch.int16)):
            raise RuntimeError("e2e outputs differ from the device outputs")

    # ---------------- CPU baseline (rank 0, N = 1)
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu:
        torch.set_num_threads(host_cores())
        s = cpu_sample(lay, a.seed, a.cpu_seats)
        rate, n, el = cpu_rate(s, L, a.cpu_seconds)
        cpu = {"value": rate, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{n} steps of all {L} layers for {s['n']} of {B} seats in {el:.1f} s (append + page gather "
                         f"+ Talker._attn_ref restated, fp32 torch CPU); seat-steps/s = sampled seats / step time"}

    for g in graphs:
        del g
    graphs.clear()
    # ---------------- the other configurations, timed briefly in the same run (1 GPU), outside the timed region
    other = None
    if rank == 0 and world == 1 and not a.no_aux:
        import copy
        other = {}
        for w in ("c3", "c4", "prefill", "ring"):
            b = copy.copy(a)
            b.workload, b.steps, b.warmup = w, 20, 3
            r = bench_aux(b)
            other[w] = {k: v for k, v in r.items() if k not in ("workload", "reference_a100", "peak_hbm_gbs",
                                                                "peak_source")}
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
                "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic (seeded, BASELINE config 2 shapes; K/V N(0,1)*0.5)",
                "config": config_dict(a, world), "gpu_launches": a.steps * L, "roofline": roof,
                "e2e": e2e, "cpu_baseline": cpu, "clocks": clk,
                "hbm_gbs_per_gpu": achieved, "hbm_frac_of_peak": achieved / peak, "other_configs": other}
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
