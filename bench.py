#!/usr/bin/env python
"""Benchmark: batched greedy decode of the Pebble-25M architecture on B200.

Workload (one "step"): krk_generate_greedy over the rank's sequences --
prompts of 128 token ids ~U[0,2048) (numpy seed 1), 256 new tokens each with
EOS ignored, context 2048 -- on random-init seed-0 weights (the real
checkpoint is not distributed).  By default 1024 sequences in total are split
evenly over the N GPUs (strong scaling: 128 per GPU at N=8); `--seqs S` runs S
sequences per GPU instead (weak scaling).  No collectives on the data path;
throughput = generated tokens of all ranks / max over ranks of the time.

  value  device time of the generate calls from the state reset to the last
         pick (the prompts and the call's tables are already on the device);
         the timed loop runs with whole-call events only (no per-kernel events)
  e2e    the same calls timed end to end on the model stream, including the
         pinned-host -> device prompt copy and the device -> host token read
  roofline  the decode SSD update's per-launch rate in a separate profiled
         call after the timed region (same configuration, per-kernel events)
  c1     batch 1, a 32-token prompt, 64 greedy tokens through the same call
         (the reference's own use case), with the oracle's batch-1 rate
  kernels  per-kernel HBM throughput of the fused layer kernels at their
         benchmark shapes (gated norm [16384,512], RoPE+KV+attention
         [64,8,2048,64], conv+SSD step [256,16,64,128], conv+SSD scan T=2048)

`--impl reference` times the CPU restatement of the reference path (the Rust
crate cannot be built on these machines) on the host cores; it loads only the
oracle's library and numpy, never the CUDA library.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HID, VOC, INTER, DIP, DI, QKV = 608, 2048, 2432, 2707, 1216, 1824
MAMBA_LAYERS, ATTN_LAYERS = 6, 2
SSD_STATE_FLOATS = 19 * 64 * 128
SSD_TRAFFIC_PER_SEQ = 263.7e6 / 256  # measured: DRAM bytes per sequence of one ssd_step launch
METRIC = "decode tokens/s (batched greedy, Pebble-25M architecture, fp32)"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--total-seqs", type=int, default=1024,
                    help="sequences split evenly over the GPUs (strong scaling, the default)")
    ap.add_argument("--seqs", type=int, default=0, help="sequences per GPU instead (weak scaling)")
    ap.add_argument("--prompt-len", type=int, default=128)
    ap.add_argument("--new-tokens", type=int, default=256)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--no-kernels", action="store_true", help="skip the per-kernel table")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample budget")
    ap.add_argument("--kernels-only", action="store_true", help="only the per-kernel table")
    ap.add_argument("--scan-t", type=int, default=2048, help="tokens of the conv+SSD scan case")
    ap.add_argument("--decode-streams", type=int, default=3, help="parts of the decode batch on their own streams")
    ap.add_argument("--no-c1", action="store_true", help="skip the batch-1 (C1) line")
    ap.add_argument("--no-step-graphs", action="store_true",
                    help="launch each decode step kernel by kernel instead of replaying its CUDA graph")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.seqs > 0:
        args.scaling, args.seqs_per_gpu = "weak", args.seqs
    else:
        if args.total_seqs % world:
            ap.error(f"--total-seqs {args.total_seqs} does not split evenly over {world} GPUs")
        args.scaling, args.seqs_per_gpu = "strong", args.total_seqs // world
    args.world = world
    return args


# ----------------------------------------------------------------- peaks / clocks
def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, dev: int):
        self.dev, self.proc, self.lines = dev, None, []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 7:
                continue
            try:
                sm.append(float(p[0]))
                mx = float(p[1])
            except ValueError:
                continue
            for n, v in zip(names, p[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- algorithmic work
def gemm_flops_per_generate(b, prompt, steps):
    per_tok = 2 * HID * (MAMBA_LAYERS * (DIP + HID * 2) + ATTN_LAYERS * (QKV + HID + 2 * INTER))
    # in_proj + out_proj (608x1216 == 1216x608) per Mamba layer; wqkv, wo, fc1, fc2 per attention layer
    lm = 2 * HID * VOC
    return b * (prompt + steps) * per_tok + b * (steps + 1) * lm


def ssd_step_bytes_per_launch(b):
    # state read + write, x/z/B/C/dt reads, y write (fp32)
    return b * 4 * (2 * SSD_STATE_FLOATS + DI + DI + 128 + 128 + 19 + DI)


def attn_decode_bytes(b, prompt, steps):
    # every decode step of both attention layers reads K and V rows 0..pos and
    # writes the new k, v row; q read and out write are 2 more rows
    rows = sum(p + 1 for p in range(prompt, prompt + steps))
    return ATTN_LAYERS * b * 4 * HID * (2 * rows + 4 * steps)


def single_stream_summary(prof, seqs, plen, steps, tokens, peak, fp32_nominal):
    """Per-kernel rates of one generate call on one stream (decode and prefill);
    shares are of the summed kernel time."""
    dev_ms = prof["device_total"][0]
    kernel_ms = sum(v[0] for k, v in prof.items() if k != "device_total")
    ssd_ms, ssd_n, ssd_seqs = prof["ssd_step"]
    ssd_gbs = ssd_step_bytes_per_launch(1) * ssd_seqs / (ssd_ms * 1e-3) / 1e9
    gemm_tf = gemm_flops_per_generate(seqs, plen, steps) / (prof["gemm"][0] * 1e-3) / 1e12
    attn_gbs = attn_decode_bytes(seqs, plen, steps) / (prof["attn_decode"][0] * 1e-3) / 1e9
    return {"tokens_per_s": tokens / (dev_ms * 1e-3),
            "ssd_step": {"achieved": round(ssd_gbs, 1), "unit": "GB/s", "frac": round(ssd_gbs / peak, 3),
                         "avg_launch_us": round(ssd_ms * 1e3 / max(ssd_n, 1), 2)},
            "gemm": {"achieved": round(gemm_tf, 2), "unit": "TFLOP/s", "frac_nominal": round(gemm_tf / fp32_nominal, 3)},
            "attn_decode": {"achieved": round(attn_gbs, 1), "unit": "GB/s", "frac": round(attn_gbs / peak, 3)},
            "time_share": {k: round(v[0] / kernel_ms, 4) for k, v in prof.items() if k != "device_total"}}


# ----------------------------------------------------------------- CPU baseline
def _oracle_model():
    """The oracle (CPU restatement of the reference path) on the seed-0 weights.
    Imports only oracle/ and the numpy helpers of krikil_rs_b200.synth; the
    package's CUDA library is loaded lazily and is never touched here."""
    import oracle as O
    from krikil_rs_b200 import synth
    threads = os.cpu_count() or 1
    O.lib.orc_set_num_threads(threads)
    return O, O.OracleModel(synth.make_weights(0)), threads


def cpu_baseline(args, budget_s: float, prompt_len=None, new_tokens=None, seed=1, start=0, _cache={}):
    """The oracle on this host's cores: whole sequences (prompt + new tokens,
    batch 1 as the reference runs), sequences start, start+1, ... of the
    workload's prompts, until the time budget is used (at least one)."""
    from krikil_rs_b200 import synth
    if "m" not in _cache:
        _cache["m"] = _oracle_model()
    O, model, threads = _cache["m"]
    plen = prompt_len or args.prompt_len
    new = new_tokens or args.new_tokens
    prompts = synth.decode_prompts(max(args.seqs_per_gpu, 64) + start, plen, seed=seed)
    t0 = time.perf_counter()
    toks, nseq = 0, 0
    while nseq == 0 or (time.perf_counter() - t0 < budget_s and start + nseq < len(prompts)):
        out, _ = O.generate_greedy(model, O.OracleState(args.ctx), prompts[start + nseq].tolist(), new, eos=None)
        toks += len(out)
        nseq += 1
    dt = time.perf_counter() - t0
    return {"value": toks / dt, "unit": "tokens/s", "cores": threads, "kind": "port", "tokens": toks, "s": dt,
            "sample": f"{nseq} sequence(s) x ({plen}-token prompt + {new} greedy tokens), batch 1, "
                      f"oracle C restatement (-O3 AVX2/FMA, OpenMP {threads} threads), {dt:.1f} s"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))
    # each step is a bounded sample of the workload (whole sequences), sized so
    # the whole run stays within a few minutes
    budget = max(2.0, min(args.cpu_seconds, 120.0 / max(args.steps, 1)))
    for i in range(args.warmup):
        cpu_baseline(args, 0.0, start=i)
    vals = [cpu_baseline(args, budget, start=args.warmup + 8 * i) for i in range(args.steps)]
    toks = sum(x["tokens"] for x in vals)
    secs = sum(x["s"] for x in vals)
    v = toks / secs
    cb = {k: vals[0][k] for k in ("unit", "cores", "kind")}
    cb["value"] = v
    cb["sample"] = (f"{args.steps} step(s), each whole sequences at batch 1 for about {budget:.0f} s "
                    f"({toks} generated tokens in {secs:.1f} s); " + vals[0]["sample"].split(", ", 1)[1])
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": secs * 1e3 / args.steps,
            "higher_is_better": True, "scaling": args.scaling,
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded prompts, random-init weights)",
            "config": workload_config(args),
            "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference Rust crate cannot be built here (no cargo); its path is timed through the "
                    "oracle's C restatement on the host cores (rank 0 only)"}
    print(json.dumps(line), flush=True)


def workload_config(args):
    return {"workload": "batched greedy decode of Pebble-25M (config.json dims), random-init seed 0",
            "seqs_total": args.seqs_per_gpu * args.world, "seqs_per_gpu": args.seqs_per_gpu,
            "prompt_len": args.prompt_len, "new_tokens": args.new_tokens,
            "ctx": args.ctx, "eos": "ignored", "prompts": "U[0,2048) numpy seed 1",
            "l2": "inputs larger than L2 (SSD state per GPU: %.2f GB, plus the KV caches)"
                  % (args.seqs_per_gpu * 6 * 19 * 64 * 128 * 4 / 1e9),
            "decode_parts": args.decode_streams, "step_graphs": not args.no_step_graphs,
            "parallelism": f"replicas x{args.world} (no collectives)"}


# ----------------------------------------------------------------- per-kernel table
def kernel_table(torch, peak, scan_t=2048):
    from krikil_rs_b200 import kernels as K, synth
    dev = torch.device("cuda")
    res = {}

    def timeit(fn, iters=10, warm=3, reps=8):
        """ms per launch: the median over iters of reps back-to-back launches
        between one pair of events (so a short kernel's time does not include
        the host's launch gaps); every operand set is larger than L2 or the
        kernel is compute-bound."""
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
        for a, b in evs:
            a.record()
            for _ in range(reps):
                fn()
            b.record()
        torch.cuda.synchronize()
        return statistics.median(a.elapsed_time(b) for a, b in evs) / reps

    def put(name, nbytes, ms, extra=None):
        gbs = nbytes / (ms * 1e-3) / 1e9
        res[name] = {"ms": round(ms, 4), "bytes": int(nbytes), "gbs": round(gbs, 1), "frac": round(gbs / peak, 3)}
        if extra:
            res[name].update(extra)

    # projections at the decode shapes of one 1024-sequence step (nominal FP32 peak)
    fp32_peak = 148 * 128 * 2 * 1.965e9
    g = torch.Generator(device=dev).manual_seed(0)
    # bring the clocks up from idle before the first timing (about 0.5 s of work)
    a = torch.randn(608, 1024, device=dev, generator=g)
    wt = torch.randn(608, 2720, device=dev, generator=g)
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < 0.5:
        for _ in range(20):
            K.gemm(a, wt)
        torch.cuda.synchronize()
    for name, m, n, kd, epi, fm in (("in_proj", 1024, 2720, 608, 0, False), ("fc2", 1024, 608, 2432, 1, True)):
        a = torch.randn(kd, m, device=dev, generator=g)
        wt = torch.randn(kd, n, device=dev, generator=g)
        c = torch.zeros((n, m) if fm else (m, n), device=dev)
        ms = timeit(lambda: K.gemm(a, wt, epilogue=epi, out_fm=fm, c=c))
        fl = 2 * m * n * kd
        res[f"gemm_{name}[{m}x{n}x{kd}]"] = {"ms": round(ms, 4), "tflops": round(fl / (ms * 1e-3) / 1e12, 2),
                                            "fp32_frac_nominal": round(fl / (ms * 1e-3) / fp32_peak, 3)}
        del a, wt, c

    # The three inputs (100.6 MB) are smaller than L2, so back-to-back launches
    # rotate over four copies (537 MB): no launch finds its operands cached.
    x, z, r, w = (torch.from_numpy(a).to(dev) for a in synth.fused_norm_inputs())
    sets = [(x, z, r, torch.empty_like(x))] + [(x.clone(), z.clone(), r.clone(), torch.empty_like(x)) for _ in range(3)]
    turn = [0]

    def c2():
        xs, zs, rs, ys = sets[turn[0] % len(sets)]
        turn[0] += 1
        K.gated_rmsnorm_residual(xs, zs, rs, w, 1e-5, ys)
    put("gated_rmsnorm_residual[16384,512]", 4 * x.numel() * 4 + w.numel() * 4, timeit(c2))
    del x, z, r, sets

    q, k, v, pos, kc, vc = synth.attn_decode_inputs()
    q, k, v, kc, vc = (torch.from_numpy(a).to(dev) for a in (q, k, v, kc, vc))
    posd = torch.from_numpy(pos).to(dev)
    work = torch.empty(K.attn_work_floats(64, 8, 64, 2048, 64), device=dev)
    out = torch.empty_like(q)
    nb = int(sum((int(p) + 1) * 8 * 64 * 4 * 2 for p in pos) + 64 * 8 * 64 * 4 * 6)
    ms = {sp: timeit(lambda: K.rope_kv_attn_decode(q, k, v, kc, vc, posd, split=sp, work=work, out=out))
          for sp in (0, 64, 128, 256, 384, 512)}  # 0: the cluster kernel (one launch, no scratch)
    best = min(ms, key=ms.get)
    put("rope_kv_attn_decode[64,8,2048,64]", nb, ms[best],
        {"split": best, "ms_by_split": {str(k): round(v, 4) for k, v in ms.items()}})
    del kc, vc

    xs, bm, cm, dt, cs, ssm = synth.conv_ssd_inputs(256, 1)
    cw, cb, dtb, an, dsk = (torch.from_numpy(a).to(dev) for a in synth.conv_ssd_params())
    xs, bm, cm, dt = (torch.from_numpy(np.ascontiguousarray(a[:, 0])).to(dev) for a in (xs, bm, cm, dt))
    cs, ssm = torch.from_numpy(cs).to(dev), torch.from_numpy(ssm).to(dev)
    ys = torch.empty((256, 1024), device=dev)
    nb = 2 * ssm.numel() * 4 + 2 * cs.numel() * 4 + (xs.numel() + bm.numel() + cm.numel() + dt.numel()) * 4 + \
        ys.numel() * 4
    put("conv_ssd_step[256,16,64,128]", nb,
        timeit(lambda: K.conv_ssd_step(xs, bm, cm, dt, cs, cw, cb, ssm, dtb, an, dsk, ys)))

    T = scan_t
    xs, bm, cm, dt, cs0, ssm0 = synth.conv_ssd_inputs(256, T, seed=5, state_scale=0.0)
    xs, bm, cm, dt = (torch.from_numpy(a).to(dev) for a in (xs, bm, cm, dt))
    cs, ssm = torch.from_numpy(cs0).to(dev), torch.from_numpy(ssm0).to(dev)
    yt = torch.empty((256, T, 1024), device=dev)
    nb = (xs.numel() + yt.numel() + bm.numel() + cm.numel() + dt.numel()) * 4 + 2 * ssm.numel() * 4
    ms = timeit(lambda: K.conv_ssd_scan(xs, bm, cm, dt, cs, cw, cb, ssm, dtb, an, dsk, yt), iters=3, warm=1)
    flops = 256 * T * 16 * 64 * 128 * 5  # per state element per token: 2 mul + 1 add (update), mul + add (y)
    fp32_peak = 148 * 128 * 2 * 1.965e9  # nominal FP32 SIMT FLOP/s (no measured figure exists)
    put(f"conv_ssd_scan[256,{T},16,64,128]", nb, ms,
        {"tflops": round(flops / (ms * 1e-3) / 1e12, 2), "fp32_frac_nominal": round(flops / (ms * 1e-3) / fp32_peak, 3)})
    del xs, bm, cm, dt, yt
    torch.cuda.empty_cache()
    return res


# ----------------------------------------------------------------- our arm
def c1_line(args, model, peak):
    """The single-sequence workload on the device: batch 1, a 32-token prompt (ids
    ~U[0,2048), seed 0), 64 greedy tokens, context 2048, through the same
    generate call; the oracle's batch-1 rate on this host beside it."""
    import torch
    from krikil_rs_b200 import PebbleState
    from krikil_rs_b200._lib import check, lib
    plen, new, reps = 32, 64, 20
    prompt = np.random.default_rng(0).integers(0, VOC, plen).astype(np.uint32)
    st = PebbleState(model, args.ctx, batch=1)
    toks_h = torch.from_numpy(prompt.view(np.int32).copy()).pin_memory()
    lens_h = torch.full((1,), plen, dtype=torch.int32).pin_memory()
    out_h = torch.zeros((1, new), dtype=torch.int32).pin_memory()
    n_h = torch.zeros((1,), dtype=torch.int32).pin_memory()

    def gen():
        check(lib.krk_generate_greedy(model._h, st._h, toks_h.data_ptr(), lens_h.data_ptr(), new, 1.0, 0,
                                      out_h.data_ptr(), n_h.data_ptr()))
    for _ in range(3):
        gen()
    stream = torch.cuda.ExternalStream(model.stream)
    st.profile(True, per_kernel=False)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    ntok = 0
    for _ in range(reps):
        gen()
        ntok += int(n_h.sum())
    ev1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = ev0.elapsed_time(ev1)
    dev_ms = st.profile_read()["device_total"][0]
    st.profile(False)
    st.close()
    line = {"workload": "C1: batch 1, 32-token prompt, 64 greedy tokens, ctx 2048 (prefill inside the call)",
            "calls": reps, "tokens_per_s": ntok / (dev_ms * 1e-3), "e2e_tokens_per_s": ntok / (e2e_ms * 1e-3),
            "ms_per_call": e2e_ms / reps}
    if not args.no_cpu_baseline:
        cb = cpu_baseline(args, 5.0, prompt_len=plen, new_tokens=new, seed=0)
        line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
    return line


def run_ours(args):
    import torch
    import torch.distributed as dist

    world, rank = args.world, int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)

    from krikil_rs_b200 import PebbleModel, PebbleState, launch_count, replicas, synth
    from krikil_rs_b200._lib import check, lib

    # Two phases, each ended on every rank by one status exchange (the phase's
    # barrier): a rank that fails reports it there and all ranks stop together.
    group = dist if world > 1 else None
    with replicas.Phase(group):  # set-up and warm-up
        peak, peak_kind = measured_peaks()
        path = synth.weights_file(0)
        model = PebbleModel.load_safetensors(path, device=local)
        seqs, plen, new = args.seqs_per_gpu, args.prompt_len, args.new_tokens
        prompts = replicas.shard(synth.decode_prompts(world * seqs, plen, seed=1), world, rank)
        state = PebbleState(model, args.ctx, batch=seqs)
        state.set_decode_streams(args.decode_streams)
        state.set_step_graphs(not args.no_step_graphs)

        # pinned host buffers for the end-to-end calls
        toks_h = torch.from_numpy(np.ascontiguousarray(prompts.reshape(-1).view(np.int32))).pin_memory()
        lens_h = torch.full((seqs,), plen, dtype=torch.int32).pin_memory()
        out_h = torch.zeros((seqs, new), dtype=torch.int32).pin_memory()
        n_h = torch.zeros((seqs,), dtype=torch.int32).pin_memory()

        def generate():
            check(lib.krk_generate_greedy(model._h, state._h, toks_h.data_ptr(), lens_h.data_ptr(), new, 1.0, 0,
                                          out_h.data_ptr(), n_h.data_ptr()))

        for _ in range(args.warmup):
            generate()
        stream = torch.cuda.ExternalStream(model.stream)
        # the timed loop: whole-call device brackets only (no per-kernel events)
        state.profile(True, per_kernel=False)
        torch.cuda.synchronize()
    with replicas.Phase(group):  # the timed loop
        torch.cuda.synchronize()
        clocks = ClockSampler(local)
        clocks.start()
        try:
            l0 = launch_count()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record(stream)
            gen_tokens = 0
            for _ in range(args.steps):
                generate()
                gen_tokens += int(n_h.sum())
            ev1.record(stream)
            torch.cuda.synchronize()
            launches = launch_count() - l0
        finally:
            clk = clocks.stop()
        e2e_ms = ev0.elapsed_time(ev1)
        dev_ms = state.profile_read()["device_total"][0]
        state.profile(False)
    (e2e_ms, dev_ms), total_tokens = replicas.reduce_timings(dist, "cuda", [e2e_ms, dev_ms], gen_tokens)
    if world > 1:
        dist.barrier()
    expect = world * seqs * min(new, args.ctx - plen + 1) * args.steps
    assert total_tokens == expect, (total_tokens, expect)

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    # After the timed region: one call with per-kernel events in the same
    # configuration (the kernels' rates beside the other decode parts), and one
    # with the decode on a single stream (each kernel without the others).
    state.profile(True)
    generate()
    prof = state.profile_read()
    state.profile(False)
    state.set_decode_streams(1)
    state.profile(True)
    generate()
    prof1 = state.profile_read()
    state.profile(False)
    state.set_decode_streams(args.decode_streams)

    steps_per_gen = min(new, args.ctx - plen)
    # Per-class times are kernel times on their own stream; a decode batch of
    # 256+ sequences runs as concurrent parts, so these are per-launch rates
    # under the other parts' load, and the shares are of summed kernel time.
    # dominant HBM kernel: the decode SSD update
    ssd_ms, ssd_n, ssd_seqs = prof["ssd_step"]
    ssd_bytes = ssd_step_bytes_per_launch(1) * ssd_seqs
    ssd_gbs = ssd_bytes / (ssd_ms * 1e-3) / 1e9
    gemm_ms, gemm_n, _ = prof["gemm"]
    gemm_flops = gemm_flops_per_generate(seqs, plen, steps_per_gen)
    attn_ms, attn_n, _ = prof["attn_decode"]
    attn_bytes = attn_decode_bytes(seqs, plen, steps_per_gen)
    kernel_ms = sum(v[0] for k, v in prof.items() if k != "device_total")
    share = {k: round(v[0] / kernel_ms, 4) for k, v in prof.items() if k != "device_total"}
    fp32_tflops_nominal = 148 * 128 * 2 * 1.965e9 / 1e12  # 148 SMs x 128 FP32 lanes x FMA x 1965 MHz
    gemm_tflops = gemm_flops / (gemm_ms * 1e-3) / 1e12 if gemm_ms else 0.0
    # whole-call HBM floor: SSD state read + write per sequence, layer and step
    # (prefill scan and decode) and the decode attention's K/V reads
    call_bytes = ssd_step_bytes_per_launch(seqs) * MAMBA_LAYERS * steps_per_gen + attn_bytes
    call_ms = dev_ms / args.steps

    line = {
        "metric": METRIC,
        "value": total_tokens / (dev_ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": call_ms,
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded prompts, random-init weights)",
        "config": workload_config(args),
        "e2e": {"value": total_tokens / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": int(toks_h.numel() * 4 + lens_h.numel() * 4),
                "d2h_bytes_per_step": int(out_h.numel() * 4 + n_h.numel() * 4 + seqs * 4 + 4),
                "ms_per_step": e2e_ms / args.steps},
        "roofline": {"kernel": "ssd_step (decode SSD update + gate)", "bound": "hbm",
                     "achieved": round(ssd_gbs, 1), "peak": peak, "unit": "GB/s", "frac": round(ssd_gbs / peak, 3),
                     # ncu DRAM read + write of the model's ssd_step per decode sequence
                     # (1.030 MB; 256-sequence launches), scaled to this launch size
                     "traffic": int(SSD_TRAFFIC_PER_SEQ * ssd_seqs / max(ssd_n, 1)),
                     "traffic_source": "ncu dram__bytes_read+write, 256-sequence launches, scaled",
                     "peak_kind": peak_kind,
                     "measured": "CUDA events around each launch on its stream, in one profiled call after the "
                                 "timed region with the timed configuration",
                     "note": "per-launch rate while the other decode parts' kernels share the GPU; "
                             "see single_stream for the same kernel without them",
                     "algorithmic_bytes_per_launch": int(ssd_bytes / max(ssd_n, 1)),
                     "launches": ssd_n, "avg_launch_us": round(ssd_ms * 1e3 / max(ssd_n, 1), 2),
                     "frac_single_stream": None},
        "roofline_call": {"what": "whole generate call against its HBM floor (SSD state r+w of every decode "
                                  "step, decode K/V reads)",
                          "bytes": int(call_bytes), "ms": round(call_ms, 2),
                          "achieved": round(call_bytes / (call_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                          "frac": round(call_bytes / (call_ms * 1e-3) / 1e9 / peak, 3)},
        "roofline_gemm": {"kernel": "gemm_lane8 (fp32 SIMT projections)", "bound": "fp32",
                          "achieved": round(gemm_tflops, 2), "unit": "TFLOP/s",
                          "peak_nominal": round(fp32_tflops_nominal, 1),
                          "frac_nominal": round(gemm_tflops / fp32_tflops_nominal, 3),
                          "launches": gemm_n},
        "roofline_attn": {"kernel": "attn_decode", "bound": "hbm",
                          "achieved": round(attn_bytes / (attn_ms * 1e-3) / 1e9, 1) if attn_ms else None,
                          "unit": "GB/s", "launches": attn_n},
        "single_stream": single_stream_summary(prof1, seqs, plen, steps_per_gen,
                                               seqs * min(new, args.ctx - plen + 1), peak, fp32_tflops_nominal),
        "time_share": share,
        "kernel_ms_over_device_ms": round(kernel_ms / prof["device_total"][0], 3),
        "gpu_launches": launches,
        "clocks": clk,
    }
    line["roofline"]["frac_single_stream"] = line["single_stream"]["ssd_step"]["frac"]
    if world == 1:
        if not args.no_c1:
            line["c1"] = c1_line(args, model, peak)
        if not args.no_kernels:
            line["kernels"] = kernel_table(torch, peak, args.scan_t)
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = {k: v for k, v in cpu_baseline(args, args.cpu_seconds).items()
                                    if k not in ("tokens", "s")}
    print(json.dumps(line), flush=True)
    state.close()
    model.close()
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse_args()
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args)
    elif args.kernels_only:
        import torch
        peak, kind = measured_peaks()
        print(json.dumps({"kernels": kernel_table(torch, peak, args.scan_t), "peak_gbs": peak, "peak_kind": kind}))
    else:
        from krikil_rs_b200.replicas import ReplicaFailure
        try:
            run_ours(args)
        except ReplicaFailure as e:
            # every rank raised it at the same exchange: rank 0 reports, all end
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"metric": METRIC, "error": "replica failure",
                                  "failed_ranks": {str(r): m for r, m in sorted(e.failed.items())}}))
            import torch.distributed as dist
            if dist.is_available() and dist.is_initialized():
                dist.destroy_process_group()
            sys.exit(1)


if __name__ == "__main__":
    main()
