"""Benchmark of the B200 Whisper decoder token loop.

One "step" is one whole Decode of the batch: cross K/V precompute for every
utterance, then the token loop (224 steps, beam 5 by default) on the GPU.
Workload (default): BASELINE.json configs[4], large-v3-shaped decoder
(d=1280, 32 layers, 20 heads, vocab 51866), Q8_0 weights from seeded
N(0, 0.02), a batch of 64 utterances with synthetic N(0,1) encoder outputs
[1500, 1280], beam 5, 224 steps (EOT suppressed so every utterance runs the
full length), CORRECT-mode decoding. With N GPUs (torchrun) the 64
utterances are sharded over the ranks (64/N each, rank r takes utterances
r, r+N, ...): strong scaling of the one batch, no collective on the token
loop. `--weak` instead gives every rank its own full batch.

  value : decoder tokens/s of the whole job (utterance-steps/s summed over
          all GPUs, beams not counted), inputs resident in HBM, device time
          from CUDA events on each job's stream, max over ranks
  e2e   : same metric through the public C-ABI job API with pinned host
          encoder outputs uploaded and tokens read back every decode
  --impl reference : the CPU restatement of whisper.go's decoder (oracle),
          timed on the host cores, on a bounded sample of the same workload
"""
import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "whisper.go_b200"))

CONFIGS = {
    1: dict(name="tiny.en-shaped Q8_0 greedy", V=51864, d=384, L=4, H=6, qtype="Q8_0", beam=1, U=1),
    2: dict(name="base-shaped Q4_0 greedy", V=51865, d=512, L=6, H=8, qtype="Q4_0", beam=1, U=1),
    3: dict(name="small-shaped Q5_1 beam5", V=51865, d=768, L=12, H=12, qtype="Q5_1", beam=5, U=1),
    4: dict(name="medium-shaped Q5_0 beam5 x8", V=51865, d=1024, L=24, H=16, qtype="Q5_0", beam=5, U=8),
    5: dict(name="large-v3-shaped Q8_0 beam5 x64", V=51866, d=1280, L=32, H=20, qtype="Q8_0", beam=5, U=64),
}
PROMPT = [50258, 50259, 50357, 50363]
METRIC = "decoder tokens/s per GPU (large-v3 Q8_0, beam 5); % of HBM roofline"  # BASELINE.json metric
T_ENC, STEPS_PER_DECODE, SEED = 1500, 224, 20261201


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=5)
    ap.add_argument("--utterances", type=int, default=0,
                    help="utterances of the batch (default: the config's); sharded over the GPUs unless --weak")
    ap.add_argument("--weak", action="store_true",
                    help="weak scaling: every GPU decodes its own --utterances (default: one batch sharded)")
    ap.add_argument("--tokens", type=int, default=STEPS_PER_DECODE)
    ap.add_argument("--mode", default="correct", choices=["correct", "ref_compat"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-steps", type=int, default=2)
    ap.add_argument("--jobs", type=int, default=1,
                    help="concurrent decode jobs per GPU, each with its own stream and host thread, "
                         "splitting the GPU's utterances")
    ap.add_argument("--layers", type=int, default=0,
                    help="decoder layers (default: the config's); fewer only for small profiler captures")
    ap.add_argument("--only-class", default="",
                    help="profiler captures: start one decode job, launch only this kernel class "
                         "(wgdec.KCLASS: logits, cross_attn, self_attn, step, ...) --steps times, print nothing else")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def utterance_ids(rank, world, U, weak=False):
    """Global ids of the utterances one rank decodes (no data-path collective).

    Strong scaling (default): the batch of U utterances is sharded round-robin,
    rank r taking r, r + world, ... Weak scaling: every rank decodes its own U.
    """
    if weak:
        return [rank * U + u for u in range(U)]
    return list(range(rank, U, world))


class Dist:
    """torch.distributed plumbing: barrier, max and sum over ranks (timing only;
    nccl on GPUs, gloo when no CUDA device is visible)."""

    def __init__(self, world, local, backend=None, timeout_s=900):
        self.world = world
        self.pg = None
        if world > 1:
            import datetime
            import torch
            import torch.distributed as td
            backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
            if backend == "nccl":
                torch.cuda.set_device(local)
                td.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s),
                                      device_id=torch.device("cuda", local))
                self.device = "cuda:%d" % local
            else:
                td.init_process_group("gloo", timeout=datetime.timedelta(seconds=timeout_s))
                self.device = "cpu"
            self.td, self.torch = td, torch
            self.pg = True

    def barrier(self):
        if self.pg:
            self.td.barrier()

    def max(self, x):
        if not self.pg:
            return x
        t = self.torch.tensor([float(x)], device=self.device, dtype=self.torch.float64)
        self.td.all_reduce(t, op=self.td.ReduceOp.MAX)
        return float(t.item())

    def sum(self, x):
        if not self.pg:
            return x
        t = self.torch.tensor([float(x)], device=self.device, dtype=self.torch.float64)
        self.td.all_reduce(t, op=self.td.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.pg:
            self.td.destroy_process_group()


class Clocks:
    """nvidia-smi samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), "--query-gpu=" + self.FIELDS,
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.th.join(timeout=2)
        sm, mx, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
                power.append(float(r[3]))
            except ValueError:
                continue
            for n, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None}


# dram__bytes_read.sum + dram__bytes_write.sum per launch of each kernel class
# on the default workload (config 5, 64 utterances per GPU, 32 layers), taken
# from one ncu capture each, not measured in every run:
#   gemv       mean of the six token-loop GEMM shapes, profiles/gemm_tc_large_v3.md
#   cross_attn profiles/cross_attn_stream_large_v3.md
#   self_attn  profiles/attn_simt_self_large_v3.md
#   logits     profiles/logits_gemm_large_v3.md
# Other workloads report None (no capture covers them).
TRAFFIC = {"gemv": 6.19e6, "cross_attn": 500.6e6, "self_attn": 375.8e6, "logits": 154.7e6}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


def cpu_baseline(model, cfg, U, args, n_ctx, threads):
    """The oracle (CPU restatement of the reference decoder) on a bounded sample."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle  # test infrastructure: the timed CPU baseline only
    import wgdec
    params = wgdec.DecoderParams(prompt=PROMPT, beam_size=cfg["beam"], max_tokens=args.tokens,
                                 mode=wgdec.MODE_REF_COMPAT, suppress_eot=True)
    n_utt = min(U, threads)
    sec, toks = oracle.bench_steps(model, n_utt, T_ENC, params, args.cpu_sample_steps, threads)
    return {"value": toks / sec if sec > 0 else None, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": "%d utterances x %d token steps (beam %d, REF_COMPAT arithmetic, GEMVs serial per "
                      "hypothesis as in the reference, cross K/V cached) on %d threads: %.1f s"
                      % (n_utt, args.cpu_sample_steps, cfg["beam"], threads, sec)}


def run_reference(args, cfg, rank, world):
    if rank != 0:
        return 0
    import wgdec
    threads = os.cpu_count() or 1
    model = wgdec.SyntheticModel(cfg["V"], cfg["d"], cfg["H"], cfg["L"], 448, cfg["qtype"], seed=SEED)
    U = args.utterances or cfg["U"]
    vals = []
    for i in range(args.warmup + args.steps):
        cb = cpu_baseline(model, cfg, U, args, 448, threads)
        if i >= args.warmup:
            vals.append(cb)
    v = statistics.median([c["value"] for c in vals])
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak" if args.weak else "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random-init weights, N(0,1) encoder)",
            "config": {"workload": "config %d: %s, tokens/s extrapolated from %d token steps of %d utterances "
                                   "on the host cores" % (args.config, cfg["name"], args.cpu_sample_steps,
                                                          min(U, threads)),
                       "utterances": U, "beam": cfg["beam"], "tokens": args.tokens,
                       "sample_token_steps": args.cpu_sample_steps},
            "cpu_baseline": {"kind": "port", "cores": threads, "sample": vals[-1]["sample"], "value": v},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    cfg = CONFIGS[args.config]
    rank, world, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, cfg, rank, world)
    import numpy as np
    import wgdec
    dist = Dist(world, local)
    U_batch = args.utterances or cfg["U"]
    ids = utterance_ids(rank, world, U_batch, args.weak)
    if not ids:
        raise SystemExit("bench: %d utterances cannot be sharded over %d GPUs (use --weak)" % (U_batch, world))
    U = len(ids)  # this rank's utterances
    if args.layers:
        cfg = dict(cfg, L=args.layers)
    mode = wgdec.MODE_CORRECT if args.mode == "correct" else wgdec.MODE_REF_COMPAT
    model = wgdec.SyntheticModel(cfg["V"], cfg["d"], cfg["H"], cfg["L"], 448, cfg["qtype"], seed=SEED)
    dec = wgdec.WhisperDecoder(model, devices=[local])
    # encoder outputs of this rank's utterances, in pinned host memory
    import torch
    host = torch.empty((U, T_ENC, cfg["d"]), dtype=torch.float32, pin_memory=True)
    hnp = host.numpy()
    for u, uid in enumerate(ids):
        hnp[u] = model.encoder_output(uid, T_ENC)
    encs = [hnp[u] for u in range(U)]
    params = wgdec.DecoderParams(prompt=PROMPT, beam_size=cfg["beam"], max_tokens=args.tokens, mode=mode,
                                 suppress_eot=True)
    # J concurrent jobs split the utterances; each has its own stream, CUDA
    # graph and workspace, and a host thread drives it, so the kernels of one
    # fill the GPU while the other's kernels drain
    J = max(1, min(args.jobs, U))
    shares = [U // J + (1 if j < U % J else 0) for j in range(J)]
    offs = [sum(shares[:j]) for j in range(J)]
    jobs = [wgdec.Job(dec, shares[j], T_ENC, params) for j in range(J)]
    for j in range(J):
        jobs[j].upload(encs[offs[j]:offs[j] + shares[j]])  # resident in HBM before the timed region
    job = jobs[0]

    def run_all(fn):
        if J == 1:
            fn(jobs[0])
            return
        import threading
        errs = []

        def body(jb):
            try:
                fn(jb)
            except Exception as ex:  # re-raised on the main thread
                errs.append(ex)
        ts = [threading.Thread(target=body, args=(jb,)) for jb in jobs]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        if errs:
            raise errs[0]

    if args.only_class:  # one kernel class on its own, for an ncu capture of just its launches
        jobs[0].start()
        for _ in range(args.steps):
            jobs[0].time_kernel(args.only_class, iters=1)
        for jb in jobs:
            jb.close()
        dec.close()
        dist.close()
        return 0

    def decode_once():
        for jb in jobs:
            jb.start()
        run_all(lambda jb: jb.run())

    for _ in range(args.warmup):
        decode_once()
    dist.barrier()
    clocks = Clocks(local)
    clocks.start()
    launches0 = wgdec.kernel_launch_count()
    t_wall = time.perf_counter()
    for jb in jobs:
        jb.timer_start()
    for _ in range(args.steps):
        decode_once()
    # device time of each job's stream; with several jobs the region spans
    # from the first start to the last stop, so also take the host wall clock
    ms = max(jb.timer_stop() for jb in jobs)
    if J > 1:
        ms = max(ms, (time.perf_counter() - t_wall) * 1e3)
    launches = wgdec.kernel_launch_count() - launches0
    clk = clocks.stop()
    tokens_per_decode = 0.0
    rows = 0
    for jb in jobs:
        toks, lens, _ = jb.result()
        tokens_per_decode += float(np.sum(lens - len(PROMPT)))
        rows += jb.stats()[1]
    dist.barrier()
    ms_max = dist.max(ms)
    total_tokens = dist.sum(tokens_per_decode * args.steps)
    value = total_tokens / (ms_max / 1e3)

    # roofline: per-class device time of one step's launches (CUDA events on the job stream)
    peak, peak_kind = peaks()
    classes = {}
    steps_done, _, _ = job.stats()
    # the kernel classes a token step runs: at <= 16 rows all layers are one
    # persistent kernel ("step"), else separate matmul / attention kernels
    step_kernel = job.uses_step_kernel()
    main = ("step", "logits") if step_kernel else ("gemv", "self_attn", "cross_attn", "logits")
    per_step_launches = {"gemv": 6 * cfg["L"], "self_attn": cfg["L"], "cross_attn": cfg["L"], "logits": 1, "step": 1}
    for k in main:
        t, b = job.time_kernel(k, iters=3)
        classes[k] = {"ms_per_launch": t, "bytes_per_launch": b, "gbs": b / (t * 1e6) if t > 0 else None,
                      "ms_per_step": t * per_step_launches[k]}
    for k in ("precompute",) if step_kernel else ("qkv", "self_out", "cross_q", "cross_out", "mlp0", "mlp2",
                                                  "precompute"):
        t, b = job.time_kernel(k, iters=3)
        classes[k] = {"ms_per_launch": t, "bytes_per_launch": b, "gbs": b / (t * 1e6) if t > 0 else None,
                      "ms_per_step": t * (cfg["L"] if k != "precompute" else 1.0 / max(steps_done, 1))}
    dom = max(main, key=lambda k: classes[k]["ms_per_step"])
    default_workload = (args.config == 5 and len(ids) == 64 and cfg["L"] == CONFIGS[5]["L"] and not step_kernel
                        and args.tokens == STEPS_PER_DECODE)
    dk = classes[dom]
    roofline = {"bound": "hbm", "kernel": dom, "achieved": dk["gbs"], "peak": peak, "unit": "GB/s",
                "frac": dk["gbs"] / peak if dk["gbs"] else None,
                "traffic": TRAFFIC.get(dom) if default_workload else None,
                "peak_kind": peak_kind, "classes": classes}
    # the north star's step roofline: quantised weight + KV bytes of one token
    # step (averaged over the decode) at 8 TB/s, against the measured step time
    n_tok, P = args.tokens, len(PROMPT)
    mean_pos = P + (n_tok - 1) / 2.0
    kv_self = rows * cfg["L"] * 2 * mean_pos * cfg["d"] * 2
    kv_cross = U * cfg["L"] * 2 * T_ENC * cfg["d"] * 2
    step_bytes = dec.weight_bytes() + kv_self + kv_cross
    step_ms = ms_max / args.steps / n_tok
    step_roofline = {"bytes_per_step": step_bytes, "peak_gbs": 8000.0, "roofline_ms": step_bytes / 8e12 * 1e3,
                     "measured_ms": step_ms, "frac": (step_bytes / 8e12 * 1e3) / step_ms,
                     "frac_of_measured_peak": (step_bytes / (peak * 1e6)) / step_ms}

    for jb in jobs:
        jb.close()  # free their KV caches before the end-to-end jobs allocate their own
    # end to end through the public API: pinned host -> device, decode, tokens back
    e2e = None
    if not args.no_e2e:
        e2e_jobs = [wgdec.Job(dec, shares[j], T_ENC, params) for j in range(J)]
        out = [None] * J

        def e2e_one(j):
            jb = e2e_jobs[j]
            jb.upload(encs[offs[j]:offs[j] + shares[j]])
            jb.start()
            jb.run()
            out[j] = jb.result()

        jobs = e2e_jobs
        run_all(lambda jb: e2e_one(e2e_jobs.index(jb)))
        dist.barrier()
        for jb in e2e_jobs:
            jb.timer_start()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            run_all(lambda jb: e2e_one(e2e_jobs.index(jb)))
        e_ms = max(jb.timer_stop() for jb in e2e_jobs)
        wall = (time.perf_counter() - t0) * 1e3
        e_ms = dist.max(max(e_ms, wall))
        d2h = dist.sum(sum(int(o[0].nbytes + o[1].nbytes + o[2].nbytes) for o in out))
        h2d = dist.sum(U * T_ENC * cfg["d"] * 4)  # encoder outputs of all ranks
        e2e = {"value": total_tokens / (e_ms / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)}
        for jb in e2e_jobs:
            jb.close()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(model, cfg, U, args, 448, os.cpu_count() or 1)

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
                "higher_is_better": True, "scaling": "weak" if args.weak else "strong", "vs_baseline": None,
                "dtype": "f16xf16->f32",
                "value_is": "whole-job decoder tokens/s summed over all %d GPU(s)" % world,
                "value_per_gpu": value / world,
                "data": "synthetic (seeded random-init weights, N(0,1) encoder outputs)",
                "config": {"workload": "config %d: %s" % (args.config, cfg["name"]), "utterances": U_batch,
                           "utterances_per_gpu": U_batch if args.weak else -(-U_batch // world),
                           "beam": cfg["beam"], "rows_per_step": rows, "tokens_per_decode": args.tokens,
                           "mode": args.mode, "kv_dtype": "f16", "t_enc": T_ENC,
                           "l2": "inputs larger than L2 (per-step KV + weights >> 126 MB)",
                           "parallelism": "dp%d (utterances, no collective)" % world,
                           "jobs_per_gpu": J},
                "roofline": roofline, "step_roofline": step_roofline, "cpu_baseline": cpu, "e2e": e2e,
                "clocks": clk,
                "gpu_launches": int(launches)}
        print(json.dumps(line), flush=True)
    dec.close()
    dist.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
