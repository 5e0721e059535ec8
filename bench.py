#!/usr/bin/env python
"""Benchmark: Qwen3-TTS continuous-batching ragged decode, audio-seconds per second.

Workload (the headline configuration): 512 requests, prompt lengths uniform in
[16, 256], target lengths uniform in [100, 1500] frames, 16-token KV pages,
at most 64 active requests per GPU, full talker + code predictor + streaming
codec decode per step, replicated bf16 weights from seed 0, requests
round-robin partitioned across the GPUs (data parallel, no collective on the
hot path).  Frames are teacher-forced with uniform codes in [0, 2048) so every
request runs exactly its target length (the sampler still runs each step).

One step = one scheduler iteration (q3t_batch_step): admit + prefill queued
requests into free slots, one frame for every active request, emit the
codec chunks that are due, retire finished requests.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
Multi-GPU: python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...
"""
import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "tts-rs_b200"))

import dp  # noqa: E402
import synthetic as S  # noqa: E402

FRAME_S = 0.08          # one frame = 1920 samples at 24 kHz
SAMPLE_RATE = 24000
METRIC = "audio-sec/sec per box (batch 64 ragged continuous batching)"
WORKLOAD = ("qwen3-tts-12hz-0.6b continuous batching: 512 requests, prompt U[16,256], "
            "target U[100,1500] frames, 16-token pages, <=64 active/GPU, talker+predictor+streaming codec")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=300)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--requests", type=int, default=512)
    p.add_argument("--max-active", type=int, default=64)
    p.add_argument("--chunk", type=int, default=16)
    p.add_argument("--left-context", type=int, default=8)
    p.add_argument("--cpu-frames", type=int, default=48, help="bounded CPU-baseline sample (frames)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-b1", action="store_true", help="skip the batch-1 talker step measurement")
    p.add_argument("--only-b1", action="store_true",
                   help="run only the batch-1 talker step (prints its JSON object; for profiling)")
    p.add_argument("--b1-steps", type=int, default=256)
    p.add_argument("--only-codec", action="store_true",
                   help="run only the T=750 codec decode measurement (prints its JSON object; for profiling)")
    p.add_argument("--codec-batches", default="1,8")
    p.add_argument("--codec-frames", type=int, default=750,
                   help="--only-codec: frames per sequence (750 = 60 s; smaller cases for ncu captures)")
    p.add_argument("--no-components", action="store_true",
                   help="skip the predictor-loop (B=1/16/64) and codec (T=750, B=1/8) measurements")
    p.add_argument("--c3-frames", type=int, default=512)
    p.add_argument("--kv-pages", type=int, default=8192, help="talker KV pool size (16-token pages)")
    p.add_argument("--no-steady", action="store_true",
                   help="time right after the warm-up steps instead of after the first retirements")
    p.add_argument("--no-drain", action="store_true", help="skip the full-workload run to completion")
    p.add_argument("--profile", action="store_true",
                   help="bracket the timed steps with cudaProfilerStart/Stop (ncu --profile-from-start off)")
    return p.parse_args()


def workload(n_req, seed=0):
    g = np.random.default_rng([seed, 2024])
    S_len = g.integers(16, 257, n_req)
    T_len = g.integers(100, 1501, n_req)
    return [(int(a), int(b)) for a, b in zip(S_len, T_len)]


def request_inputs(i, S_len, T_len, H=1024):
    g = np.random.default_rng([0, 77, i])
    prompt = (g.standard_normal((S_len, H), dtype=np.float32) * 0.5)
    trailing = (g.standard_normal((1, H), dtype=np.float32) * 0.5)
    pad = (g.standard_normal((H,), dtype=np.float32) * 0.5)
    codes = g.integers(0, 2048, size=(T_len, 16), dtype=np.int64)
    return prompt, trailing, pad, codes


# per-step algorithmic HBM bytes (weights read once per step, KV read per token)
def step_bytes(stats, cfg):
    t, p = cfg.talker, cfg.predictor
    layer = lambda c: (c.hidden * (c.n_heads + 2 * c.n_kv) * c.head_dim + c.hidden * c.n_heads * c.head_dim
                       + 3 * c.hidden * c.inter) * 2
    talker_w = t.n_layers * layer(t) + t.vocab * t.hidden * 2
    pred_w = (cfg.n_groups - 1) * (p.n_layers * layer(p) + p.vocab * p.hidden * 2)
    kv = stats["kv_tokens"] * t.n_layers * 2 * t.n_kv * t.head_dim * 2
    return talker_w + pred_w + kv


class Clocks:
    """nvidia-smi clock / throttle sampling during the timed region."""

    def __init__(self, gpu_index, out):
        self.p = None
        try:
            self.f = open(out, "w")
            self.p = subprocess.Popen(
                ["nvidia-smi", f"--id={gpu_index}",
                 "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        self.path = out

    def stop(self):
        if not self.p:
            return None
        self.p.terminate()
        self.p.wait()
        self.f.close()
        sm, mx, reasons = [], 0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_baseline(n_frames, threads=0):
    """The CPU oracle (C restatement of the reference math, OpenMP) on a
    bounded sample of the same workload: one batch-1 request (the reference
    is batch-1), 64-token prompt, n_frames teacher-forced frames, then the
    codec decode of those frames.  Returns (audio-s/s, cores, seconds)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    if threads:
        O.lib().orc_set_threads(threads)
    cfg = S.TalkerConfig()
    ot = O.OracleTalker(cfg, S.make_talker_weights(cfg))
    cc = S.CodecConfig()
    oc = O.OracleCodec(cc, S.make_codec_weights(cc))
    prompt, trailing, pad, codes = request_inputs(0, 64, n_frames + 1)
    t0 = time.perf_counter()
    g = O.OracleGenerator(ot, prompt, trailing, pad, max_new_tokens=n_frames, forced_first=int(codes[0, 0]))
    for f in range(n_frames):
        g.step(forced=codes[f])
    oc.decode(g.codes()[None])
    dt = time.perf_counter() - t0
    return n_frames * FRAME_S / dt, O.lib().orc_get_threads(), dt


def talker_b1_step(model, cfg, L=1024, steps=256, warmup=3, peak=6558.1):
    """Isolated batch-1 talker decode step (hidden ~N(0,1) in, codec-head
    logits out) against a KV cache of length L (K/V ~N(0,1) bf16), through the
    session C ABI (q3t_session_decode_embeds); device time per step from the
    library's CUDA events.  Algorithmic bytes per step: every talker weight and
    the codec head once (bf16) plus K/V of every cached position and layer."""
    c = cfg.talker
    g = np.random.default_rng([0, 31])
    k = S.bf16_bits(g.standard_normal((c.n_layers, c.n_kv, L, c.head_dim), dtype=np.float32))
    v = S.bf16_bits(g.standard_normal((c.n_layers, c.n_kv, L, c.head_dim), dtype=np.float32))
    prompt, trailing, pad = S.synthetic_talker_inputs(cfg, 1, 0)
    sess = model.session(prompt, trailing, pad, max_new_tokens=4)
    sess.load_kv(k, v, L)
    emb = g.standard_normal(c.hidden).astype(np.float32)
    us, lens = [], []
    for i in range(warmup + steps):
        sess.decode_embeds(emb)
        if i >= warmup:
            us.append(sess.last_ms() * 1e3)
            lens.append(L + i + 1)
    sess.close()
    layer = (c.hidden * (c.n_heads + 2 * c.n_kv) * c.head_dim + c.hidden * c.n_heads * c.head_dim
             + 3 * c.hidden * c.inter) * 2
    wbytes = c.n_layers * layer + c.vocab * c.hidden * 2
    kv_per_pos = c.n_layers * 2 * c.n_kv * c.head_dim * 2
    byt = wbytes + kv_per_pos * float(np.median(lens))
    med = float(np.median(us))
    return {"workload": f"talker decode step, batch 1, KV length {L}..{L + warmup + steps}, {steps} steps",
            "us_per_step_p50": round(med, 2), "bytes_per_step": int(byt),
            "achieved_gbs": round(byt / med / 1e3, 1), "peak_gbs": peak,
            "frac": round(byt / med / 1e3 / peak, 4)}


def predictor_loop(model, cfg, batches=(1, 16, 64), frames=512, warmup=3, peak=6558.1):
    """The 15-codebook code-predictor loop per decode frame at batch B
    (teacher-forced, 16-token prompts, greedy sampler), timed on the device as
    the frame's predictor graph (CUDA events on the batch stream).  Bytes per
    frame-step: 15 passes x the 5 predictor layers + one lm_head each (bf16),
    independent of B."""
    p = cfg.predictor
    layer = (p.hidden * (p.n_heads + 2 * p.n_kv) * p.head_dim + p.hidden * p.n_heads * p.head_dim
             + 3 * p.hidden * p.inter) * 2
    byt = (cfg.n_groups - 1) * (p.n_layers * layer + p.vocab * p.hidden * 2)
    out = {"workload": f"code predictor loop, {frames} frames per batch size, 15 codebooks x 5 layers, greedy",
           "bytes_per_frame_step": int(byt)}
    for B in batches:
        b = model.batch(max_active=B, codec_mode=0, keep_output=0)
        for i in range(B):
            prompt, trailing, pad, _ = request_inputs(10000 + i, 16, 1)
            codes = np.random.default_rng([1, i]).integers(0, 2048, (frames + warmup + 2, 16), dtype=np.int64)
            b.submit(prompt, trailing, pad, codes.shape[0], forced=codes)
        st = [b.step() for _ in range(warmup + frames)]
        b.close()
        full = [s for s in st[warmup:] if s["active"] == B and s["prefill_tokens"] == 0]
        pm = [s["predictor_ms"] for s in full]
        tm = [s["talker_ms"] for s in full]
        med = float(np.median(pm))
        out[f"B{B}"] = {"predictor_ms_per_frame_p50": round(med, 4), "talker_ms_per_frame_p50": round(float(np.median(tm)), 4),
                        "achieved_gbs": round(byt / med / 1e6, 1), "frac": round(byt / med / 1e6 / peak, 4)}
    out["peak_gbs"] = peak
    return out


def codec_flops_per_frame(c, T):
    """Multiply-adds x 2 of one 12.5 Hz frame through the speech-tokenizer
    decoder (quantizer projections, pre-conv, pre-transformer with T x T
    attention, ConvNeXt upsampling, SnakeBeta wave decoder, output conv)."""
    half, D, LAT, H = c.codebook_dim // 2, c.codebook_dim, c.latent, c.hidden
    f = 2 * (2 * half * D) + 2 * 3 * D * LAT + 2 * LAT * H * 2
    nq = c.n_heads * c.head_dim
    f += c.n_layers * 2 * (H * (nq + 2 * c.n_kv * c.head_dim) + nq * H + 3 * H * c.inter + 2 * T * nq)
    steps = 1
    for r in c.up_ratios:
        steps *= r
        f += steps * 2 * (LAT * LAT + 7 * LAT + 2 * LAT * 4 * LAT)
    f += steps * 2 * 7 * LAT * c.decoder_dim
    ch = c.decoder_dim
    for r in c.rates:
        steps *= r
        f += steps * 2 * (ch * (ch // 2) * 2 + 3 * (7 + 1) * (ch // 2) ** 2)
        ch //= 2
    return f + steps * 2 * 7 * ch


def codec_decode_t750(model, cc, batches=(1, 8), T=750, reps=3, peak_tflops=1610.8):
    """Speech-tokenizer decode of T frames (60 s of audio at T = 750) at batch
    B, device time from the library's CUDA events (codes on the device ->
    samples on the device); FLOPs from the decoder shapes."""
    import q3t
    fl = codec_flops_per_frame(cc, T)
    out = {"workload": f"codec decoder, codes [B,16,{T}] uniform in [0,2048) -> 24 kHz f32 PCM",
           "gflop_per_frame": round(fl / 1e9, 3)}
    for B in batches:
        codes = np.random.default_rng([B, 750]).integers(0, 2048, (B, 16, T), dtype=np.int64)
        model.codec_decode(codes[:, :, :32])  # warm-up (workspace pools)
        ms = []
        for _ in range(reps):
            model.codec_decode(codes)
            ms.append(q3t.Model.codec_last_ms())
        med = float(np.median(ms))
        tf = fl * T * B / (med / 1e3) / 1e12
        out[f"B{B}"] = {"ms": round(med, 2), "audio_s_per_s": round(B * T * FRAME_S / (med / 1e3), 1),
                        "tflops": round(tf, 1), "frac": round(tf / peak_tflops, 4)}
    out["peak_tflops"] = peak_tflops
    out["peak_note"] = "measured bf16 dense GEMM burst peak (the codec's fp16 tensor-core rate is the same)"
    return out


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    args.steady_off = args.no_steady
    import torch
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    torch.cuda.set_device(local)
    import q3t

    cfg = S.TalkerConfig()
    cc = S.CodecConfig()
    if args.only_codec:
        model = q3t.Model(codec_cfg=cc, codec_weights=S.make_codec_weights(cc, 0), device=local)
        pk = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))).get("bf16_tflops", 1590.0) \
            if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json")) else 1590.0
        bs = tuple(int(x) for x in args.codec_batches.split(","))
        print(json.dumps(codec_decode_t750(model, cc, batches=bs, T=args.codec_frames, peak_tflops=pk)), flush=True)
        model.close()
        return
    if args.only_b1:
        model = q3t.Model(cfg, S.make_talker_weights(cfg, 0), device=local, kv_pages=128, max_active=1)
        peak = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))).get("hbm_gbs", 6650.0) \
            if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json")) else 6650.0
        print(json.dumps(talker_b1_step(model, cfg, steps=args.b1_steps, peak=peak)), flush=True)
        model.close()
        return
    model = q3t.Model(cfg, S.make_talker_weights(cfg, 0), cc, S.make_codec_weights(cc, 0), device=local,
                      kv_pages=args.kv_pages, max_active=args.max_active)
    reqs = workload(args.requests)
    mine = dp.partition(len(reqs), rank, world)
    inputs = {i: request_inputs(i, *reqs[i]) for i in mine}

    def submit(b, i):
        prompt, trailing, pad, codes = inputs[i]
        return b.submit(prompt, trailing, pad, codes.shape[0], forced=codes)

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()

    # ---------------- value: inputs resident, PCM stays on the device --------
    b = model.batch(max_active=args.max_active, codec_mode=2, chunk_frames=args.chunk,
                    left_context=args.left_context, keep_output=0)
    for i in mine:
        submit(b, i)
    def steady(step):
        """Untimed steps until the first requests retire, so a timed window
        holds the workload's mix of admissions, prompt chunks, decode frames
        and retirements rather than the initial fill (every rank takes the
        same number of steps; bounded by the longest target)."""
        n = 0
        if not args.steady_off:
            while n < 4000:
                n += 1
                if step()["retired"] > 0:
                    break
        if dist:
            t = torch.tensor([n], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            for _ in range(int(t.item()) - n):
                step()
            n = int(t.item())
        return n

    for _ in range(args.warmup):
        b.step()
    fill = steady(b.step)
    stream = torch.cuda.ExternalStream(b.stream(), device=local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # raw nvidia-smi samples of the timed region (the JSON line carries their summary)
    clocks = Clocks(local, os.path.join(os.environ.get("Q3T_BENCH_OUT", tempfile.gettempdir()), f"clocks_r{rank}.csv"))
    launches0 = q3t.kernel_launches()
    barrier()
    if args.profile:
        torch.cuda.profiler.start()
    e0.record(stream)
    t0 = time.perf_counter()
    steps = [b.step() for _ in range(args.steps)]
    e1.record(stream)
    if os.environ.get("Q3T_BENCH_STEP_LOG"):
        with open(os.environ["Q3T_BENCH_STEP_LOG"], "w") as f:
            json.dump(steps, f)
    barrier()
    if args.profile:
        torch.cuda.profiler.stop()
    wall = time.perf_counter() - t0
    launches = q3t.kernel_launches() - launches0
    ck = clocks.stop()
    dev_s = e0.elapsed_time(e1) / 1e3
    samples = sum(s["samples"] for s in steps)
    frames = sum(s["frames"] for s in steps)
    step_ms = [s["device_ms"] for s in steps]
    # the roofline's unit is the decode frame (the predictor and talker graphs,
    # CUDA events on the batch stream around them) of the steps without prompt
    # tokens; the streaming codec runs beside it on its own stream
    pure = [s for s in steps if s["prefill_tokens"] == 0 and s["active"] > 0]
    decode_ms = [s["predictor_ms"] + s["talker_ms"] for s in pure]
    bytes_ = [step_bytes(s, cfg) for s in pure]
    window = {"fill_steps": fill, "admissions": int(sum(s["admitted"] for s in steps)),
              "prompt_tokens": int(sum(s["prefill_tokens"] for s in steps)),
              "steps_with_prompt_tokens": int(sum(1 for s in steps if s["prefill_tokens"] > 0)),
              "retirements": int(sum(s["retired"] for s in steps))}
    b.close()

    # ---------------- drain: the whole workload of this rank to completion ---
    drain = None
    if not args.no_drain:
        bd = model.batch(max_active=args.max_active, codec_mode=2, chunk_frames=args.chunk,
                         left_context=args.left_context, keep_output=0)
        for i in mine:
            submit(bd, i)
        streamd = torch.cuda.ExternalStream(bd.stream(), device=local)
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        d0.record(streamd)
        std = []
        while True:
            std.append(bd.step())
            if bd.pending() == (0, 0):
                break
        d1.record(streamd)
        barrier()
        bd.close()
        drain = {"_samples": sum(s["samples"] for s in std), "_dev_s": d0.elapsed_time(d1) / 1e3,
                 "steps": len(std), "admissions": int(sum(s["admitted"] for s in std)),
                 "p50_step_ms": round(float(np.percentile([s["device_ms"] for s in std], 50)), 4),
                 "p99_step_ms": round(float(np.percentile([s["device_ms"] for s in std], 99)), 4)}

    # ---------------- e2e: host buffers in and out through the C ABI ---------
    e2e = None
    if not args.no_e2e:
        b2 = model.batch(max_active=args.max_active, codec_mode=2, chunk_frames=args.chunk,
                         left_context=args.left_context, keep_output=1)
        pending = list(mine)

        def top_up():
            q, a = b2.pending()
            while pending and q + a < args.max_active:
                submit(b2, pending.pop(0))
                q += 1

        for _ in range(args.warmup):
            top_up()
            b2.step()

        def step2():
            top_up()
            return b2.step()

        steady(step2)
        barrier()
        t0 = time.perf_counter()
        st2 = []
        for _ in range(args.steps):
            top_up()
            st2.append(b2.step())
        barrier()
        wall2 = time.perf_counter() - t0
        b2.close()
        e2e_samples = sum(s["samples"] for s in st2)
        e2e = {"value": None, "unit": "audio-s/s",
               "window": "the same steady-state window as value, requests submitted from host buffers as "
                         "others retire (prompt uploads inside the timed region)",
               "admissions": int(sum(s["admitted"] for s in st2)),
               "h2d_bytes_per_step": int(np.mean([s["h2d_bytes"] for s in st2])),
               "d2h_bytes_per_step": int(np.mean([s["d2h_bytes"] for s in st2])),
               "_samples": e2e_samples, "_wall": wall2}

    # ---------------- reduce over ranks (the one collective) -----------------
    red = dp.reduce_stats({"samples": (samples, "sum"), "frames": (frames, "sum"), "dev_s": (dev_s, "max"),
                           "e2e_samples": (e2e["_samples"] if e2e else 0, "sum"),
                           "e2e_wall": (e2e["_wall"] if e2e else 0.0, "max"),
                           "drain_samples": (drain["_samples"] if drain else 0, "sum"),
                           "drain_dev_s": (drain["_dev_s"] if drain else 0.0, "max")},
                          device="cuda" if dist else "cpu")
    if drain:
        drain = {"workload": f"all {len(reqs)} requests run to completion (this line: {world} GPU(s))",
                 "value": round(red["drain_samples"] / SAMPLE_RATE / red["drain_dev_s"], 3), "unit": "audio-s/s",
                 "device_s": round(red["drain_dev_s"], 3), "steps_rank0": drain["steps"],
                 "admissions_rank0": drain["admissions"], "p50_step_ms_rank0": drain["p50_step_ms"],
                 "p99_step_ms_rank0": drain["p99_step_ms"]}
    tot_samples, tot_frames, max_dev = red["samples"], red["frames"], red["dev_s"]
    e2e_tot, e2e_wall = red["e2e_samples"], red["e2e_wall"]
    value = tot_samples / SAMPLE_RATE / max_dev
    if e2e:
        e2e["value"] = round(e2e_tot / SAMPLE_RATE / e2e_wall, 3)
        e2e.pop("_samples")
        e2e.pop("_wall")

    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    b1 = c3 = c4 = None
    if rank == 0 and not args.no_b1:
        b1 = talker_b1_step(model, cfg, steps=args.b1_steps, peak=hbm_peak)
    if rank == 0 and not args.no_components:
        c3 = predictor_loop(model, cfg, frames=args.c3_frames, peak=hbm_peak)
        c4 = codec_decode_t750(model, cc, peak_tflops=peaks.get("bf16_tflops", 1590.0))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, dt = cpu_baseline(args.cpu_frames)
        cpu = {"value": round(v, 4), "unit": "audio-s/s", "cores": cores, "kind": "port",
               "sample": f"one batch-1 request, 64-token prompt, {args.cpu_frames} teacher-forced frames "
                         f"(28-layer talker + 5-layer predictor) + codec decode, {dt:.1f} s"}

    med_ms = float(np.median(decode_ms)) if decode_ms else float(np.median(step_ms))
    ach = (float(np.median(bytes_)) / 1e9) / (med_ms / 1e3) if bytes_ else None
    # DRAM bytes per decode step: the ncu-measured ratio of DRAM reads to
    # algorithmic bytes (profiles/decode_step_dram_bench64.md) times this
    # run's algorithmic bytes per step
    traffic = None
    try:
        for line in open(os.path.join(ROOT, "profiles", "decode_step_dram_bench64.md")):
            if line.startswith("traffic_ratio_to_algorithmic:") and bytes_:
                traffic = int(float(line.split(":")[1]) * float(np.median(bytes_)))
    except OSError:
        pass
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": "audio-s/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(max_dev * 1e3 / args.steps, 4),
            "p50_step_ms": round(float(np.median(step_ms)), 4),
            "p50_decode_frame_ms": round(med_ms, 4),
            "frames": int(tot_frames),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seed-0 random-init weights, teacher-forced uniform codes)",
            "config": {"workload": WORKLOAD, "requests": args.requests, "max_active_per_gpu": args.max_active,
                       "page_tokens": 16, "codec": f"streaming chunks of {args.chunk} frames, "
                       f"{args.left_context} frames left context", "parallelism": f"dp{world} (replicas)",
                       "l2_policy": "working set > L2 (talker+predictor weights 1.2 GB per step)",
                       "window": ("timed from steady state: untimed steps after the warm-up until the first "
                                  "retirements, so admissions, prompt chunks (packed into the talker passes) and "
                                  "retirements fall inside the window" if not args.steady_off
                                  else "timed right after the warm-up steps"),
                       "window_counts": window},
            "roofline": {"bound": "hbm", "unit": "GB/s",
                         "kernel": "decode frame step (CUDA graph of talker + predictor kernels)",
                         "achieved": round(ach, 1) if ach else None, "peak": hbm_peak,
                         "frac": round(ach / hbm_peak, 4) if ach else None, "traffic": traffic,
                         "traffic_unit": "bytes per decode step (ncu DRAM reads, scaled from a 64-request capture)",
                         "algorithmic_bytes": int(np.median(bytes_)) if bytes_ else None,
                         "peak_source": "measured" if "hbm_gbs" in peaks else "fallback"},
            "talker_b1": b1,
            "predictor_loop": c3,
            "codec_t750": c4,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "drain": drain,
            "gpu_launches": int(launches),
            "clocks": ck,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def reference_arm(args, rank, world):
    """The reference's CPU path: the oracle restatement of the Burn flex
    path (the Rust reference cannot be built here), all host threads,
    batch-1 as the reference is; each step = one frame of one request (plus
    its share of the codec decode at the end)."""
    if rank != 0:
        return
    n = max(1, args.steps)
    w = max(0, min(args.warmup, 3))
    v, cores, dt = cpu_baseline(n + w)
    print(json.dumps({
        "metric": METRIC, "impl": "reference", "value": round(v, 4), "unit": "audio-s/s",
        "n_gpus": world, "steps": n, "warmup": w, "ms_per_step": round(dt * 1e3 / (n + w), 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seed-0 random-init weights, teacher-forced uniform codes)",
        "config": {"workload": WORKLOAD + " (CPU: one batch-1 request, 64-token prompt)"},
        "cpu_baseline": {"value": round(v, 4), "unit": "audio-s/s", "cores": cores, "kind": "port",
                         "sample": f"{n + w} frames of one request + codec decode ({dt:.1f} s)"},
        "e2e": {"value": round(v, 4), "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


if __name__ == "__main__":
    main()
