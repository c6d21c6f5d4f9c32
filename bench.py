"""Benchmark: candidate-pixel decodes per second of ES training iterations on B200.

A step is one ES-phase training iteration of the benchmark's config 2 (512x512 synthetic RGB8 image,
level 0 = 512x512x1 2-bit --qat selector plane, level 1 = 128x128x2 bilinear, 24-24 MLP -> 3, population
8192 = 4096 antithetic pairs, minibatch 4096, 4 latent pairs): mlp_step + lat_step + qat_search, which is
2N M + 2K W H + sum_c 2^B_c W H = 36.7 M candidate-pixel decodes.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config C]

--impl ours (default): the CUDA backend. N > 1 (torchrun, one process per GPU): one ntcb_shard_iteration call per
iteration (neural_block_textures_b200.shard.NativeShardedES): the ES population is sharded over the ranks (each
evaluates its pairs, regenerating their noise from the counter, and sums its own ES-gradient segments), the latent
step by texel rows and the selector search by level-0 rows, and each of the three exchanges per iteration is the
library's peer-memory kernel over CUDA IPC mappings (--exchange nccl: NCCL all-gathers on the library's own
communicator; --shard-driver python: the per-phase entry points around torch.distributed all-gathers). Every rank
ends each iteration bit-identical to one GPU.
--impl reference: the reference's own CPU trainer (main.cpp compiled from source, OpenMP on every host
thread) timed on a bounded sample of the same iteration (rank 0 only).

Timing: W warm-up iterations, then the ranks are lined up (stream drained, barrier, device synchronised) and K
iterations are timed one by one with CUDA events on the trainer's stream, the L2 flushed before each outside the
events; ms_per_step is the per-rank sum / K, max over ranks (ms_per_step_median beside it). The same rules time
the FD phase, the NCCL-exchange variant (N > 1: the north star's all-gather over NCCL instead of the peer-memory
kernel) and the `cfg5` leg: the north star's scaling configuration (config 5, 2048^2, population 32768) on the same
N GPUs, so that the per-N lines carry its strong-scaling inputs next to the config-2 headline.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L2_FLUSH_BYTES = 256 << 20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)   # ~2 s timed: long enough for the 200 ms clock samples
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--fd-steps", type=int, default=100, help="FD-phase iterations timed after the ES ones (0: skip)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-cuda", action="store_true", help="skip timing the reference's own CUDA backend (oracle/_ref/ntc_ref)")
    ap.add_argument("--no-cfg5", action="store_true", help="skip the config-5 (population 32768) leg")
    ap.add_argument("--shard-driver", default="native", choices=["native", "python"],
                    help="N > 1: one library call per iteration with in-place NCCL all-gathers on the library's own communicator "
                         "(native), or the per-phase entry points around torch.distributed all-gathers (python)")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="native driver: the library's peer-memory exchange kernel over CUDA IPC (p2p) or NCCL all-gathers")
    ap.add_argument("--pop-kernel", default="tensor", choices=["tensor", "ffma"],
                    help="ES population kernel: tcgen05 3xTF32 (default) or the bit-exact packed-FP32 one")
    return ap.parse_args()


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1])); mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def reference_arm(args, world, rank):
    """The reference CPU trainer (oracle/_ref/libntc_refcpu.so, main.cpp compiled unmodified) on all host threads."""
    if world > 1 and rank != 0:
        return
    from neural_block_textures_b200 import model
    from oracle.oracle import RefSession, refcpu_available, refcpu_lib
    cfg = model.config(args.config)
    line = {"impl": "reference", "metric": "candidate-pixel decodes/s (ES training iteration)", "unit": "decodes/s",
            "higher_is_better": True, "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup}
    if not refcpu_available():
        line["unavailable"] = "oracle/_ref/libntc_refcpu.so was not built (the reference tree was absent at build time)"
        print(json.dumps(line)); return
    sess, sample_pairs, dec, cores = _ref_sample_setup(cfg)
    for _ in range(args.warmup):
        _ref_sample_step(sess, cfg, sample_pairs, 1)
    ts = []
    for k in range(args.steps):
        t0 = time.perf_counter()
        _ref_sample_step(sess, cfg, sample_pairs, 2 + k)
        ts.append(time.perf_counter() - t0)
    total = sum(ts)
    value = dec * args.steps / total
    line.update({"value": value, "ms_per_step": 1e3 * total / args.steps, "scaling": "none", "vs_baseline": None,
                 "dtype": "f32", "data": "synthetic",
                 "config": {"workload": cfg.name, "cli": cfg.cli, "sample": f"{sample_pairs} of {cfg.pairs} ES pairs per step + "
                            "the full latent step + the full selector search", "l2": "n/a (CPU)"},
                 "cpu_baseline": {"value": value, "unit": "decodes/s", "cores": cores, "kind": "reference",
                                  "sample": f"per step: MLP ES with {sample_pairs} pairs x M={cfg.batch}, latent ES K={cfg.lat_pairs}, "
                                            f"qat search; {dec / 1e6:.2f} M decodes"},
                 "e2e": {"value": value, "unit": "decodes/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
    print(json.dumps(line))


def _ref_sample_setup(cfg):
    from oracle.oracle import RefSession, refcpu_lib
    lib = refcpu_lib()
    # torchrun exports OMP_NUM_THREADS=1 to every rank; the reference CPU path gets every core this process may use.
    lib.ref_set_threads(len(os.sched_getaffinity(0)))
    cores = int(lib.ref_max_threads())
    spec = cfg.spec
    sess = RefSession(spec, cfg.target())
    z, p = spec.init_params()
    sess.set_model(z, p)
    sample_pairs = min(cfg.pairs, 256)
    d = cfg.decodes_per_iter()
    dec = 2 * sample_pairs * cfg.batch + d["latent"] + d["qat"]
    return sess, sample_pairs, dec, cores


def _ref_sample_step(sess, cfg, pairs, it):
    sess.iteration(it, pairs, cfg.batch, cfg.mlp_sigma, cfg.mlp_lr, 0, cfg.fd_h, cfg.lat_pairs, cfg.lat_sigma, cfg.lat_lr)


def cpu_baseline_leg(cfg, budget_s=12.0):
    """The reference CPU path on the host cores (rank 0, N=1), bounded to ~budget_s seconds of work."""
    from oracle.oracle import refcpu_available
    if not refcpu_available():
        return None
    sess, pairs, dec, cores = _ref_sample_setup(cfg)
    _ref_sample_step(sess, cfg, pairs, 1)
    n, t_all = 0, 0.0
    while t_all < budget_s and n < 50:
        t0 = time.perf_counter()
        _ref_sample_step(sess, cfg, pairs, 2 + n)
        t_all += time.perf_counter() - t0
        n += 1
    return {"value": dec * n / t_all, "unit": "decodes/s", "cores": cores, "kind": "reference",
            "sample": f"{n} reference CPU iterations of {cfg.name} with {pairs} of {cfg.pairs} ES pairs (+ full latent step "
                      f"and selector search): {dec / 1e6:.2f} M decodes each, {t_all:.1f} s"}


def progress_print_leg(tr, cfg, with_reference: bool, reps=5):
    """The progress print's statistics (main.cpp:4155-4205) once per print, wall clock: ntcb_print_stats on the
    device, and the reference's print path with this backend (download_model, then on the host bitrate_stats,
    mse_of of two device decodes downloaded through decode_full, latent_stats; the reference's own functions
    through oracle/_ref)."""
    spec = cfg.spec
    lb = [8] * len(spec.levels)
    tr.print_stats(lb)
    t0 = time.perf_counter()
    for _ in range(reps):
        st, _ = tr.print_stats(lb)
    out = {"device_ms": (time.perf_counter() - t0) / reps * 1e3, "mse": st.mse, "mse_q": st.mse_q, "bpp_q8": st.bpp_q8,
           "bpp_est": st.bpp_est}
    from oracle.oracle import RefSession, refcpu_available
    if not with_reference or not refcpu_available():
        return out
    sess = RefSession(spec, cfg.target())
    t_all = 0.0
    for _ in range(2):
        t0 = time.perf_counter()
        z, p = tr.download_model()
        sess.set_model(z, p)
        rw, _ = sess.mse_of(tr.decode_full())
        rs, zq = sess.bitrate_stats(8)
        rq, _ = sess.mse_of(tr.decode_full(zq))
        for l in range(min(2, len(spec.levels))):
            sess.latent_stats(l)
        t_all = time.perf_counter() - t0
    sess.close()
    out["reference_path_ms"] = t_all * 1e3
    out["reference_path"] = "download_model + host bitrate_stats / mse_of x2 / latent_stats + 2 decode_full downloads"
    out["agrees"] = bool(abs(rw - st.mse) <= 1e-12 * rw and abs(rq - st.mse_q) <= 1e-12 * rq and
                         abs(rs["bpp_q8"] - st.bpp_q8) <= 1e-12 * rs["bpp_q8"])
    return out


def ntcb_decode_leg(reps=20):
    """The .ntcb decoder at the config-5 size: a 2048 x 2048 container (--qat 2 level 0 at 1024 x 1024 x 2, 8-bit level 1
    at 256 x 256 x 4) written by the reference's own CPU trainer (oracle/_ref/ntc_cpu --write-ntcb, one iteration),
    decoded to RGB8 on the device (CUDA events over `reps` decodes, and once end to end into host memory) and by the
    reference's own CPU decoder (oracle/_ref/ntc_decode --exact --bench on every host thread)."""
    import re
    import tempfile
    import torch
    from neural_block_textures_b200 import ntcb, synth
    ref = ROOT / "oracle" / "_ref"
    if not (ref / "ntc_cpu").exists() or not (ref / "ntc_decode").exists():
        return None
    with tempfile.TemporaryDirectory() as t:
        t = Path(t)
        synth.write_png(t / "img.png", synth.synth_rgb8(2048, 2048, 5))
        r = subprocess.run([str(ref / "ntc_cpu"), str(t / "img.png"), *"--latent 1024 1024 2 --latent2 256 256 4 --filter nearest,bilinear "
                            "--qat 2 --mlp-pairs 8 --mlp-batch 1024 --iters 1 --seed 5 --rng hash --print-every 1000000 "
                            "--write-ntcb".split(), "--out", str(t / "o")], capture_output=True, text=True, timeout=600)
        if r.returncode != 0:
            return {"unavailable": "the reference trainer did not write the container"}
        data = (t / "o" / "model.ntcb").read_bytes()
        threads = len(os.sched_getaffinity(0))
        d = subprocess.run([str(ref / "ntc_decode"), str(t / "o" / "model.ntcb"), "-o", str(t / "dec"), "--exact", "--bench",
                            "--threads", str(min(threads, 64))], capture_output=True, text=True, timeout=600)
        m = re.search(r"^exact\s+(\d+)\s+[\d.]+\s+[\d.]+\s+[\d.]+\s+([\d.]+)", d.stdout, re.M)
        ref_rgb = synth.read_png(t / "dec.png") if (t / "dec.png").exists() else None
    with ntcb.NtcbDecoder(data) as dec:
        W, H = dec.info.src_w, dec.info.src_h
        out = torch.empty(W * H * 3, dtype=torch.uint8, device="cuda")
        s = torch.cuda.Stream()
        for _ in range(3):
            dec.rgb8_device(out.data_ptr(), 0, 0, s.cuda_stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.synchronize()
        e0.record(s)
        for _ in range(reps):
            dec.rgb8_device(out.data_ptr(), 0, 0, s.cuda_stream)
        e1.record(s)
        e1.synchronize()
        dev_ms = e0.elapsed_time(e1) / reps
        t0 = time.perf_counter()
        rgb = dec.rgb8()
        host_ms = (time.perf_counter() - t0) * 1e3
    line = {"workload": "2048x2048 container, --qat 2 level 0 1024x1024x2 + 8-bit level 1 256x256x4, (8, 24, 24, 3) MLP",
            "bytes": len(data), "device_ms": dev_ms, "device_mtexel_s": W * H / dev_ms / 1e3,
            "e2e_host_ms": host_ms, "e2e_host_mtexel_s": W * H / host_ms / 1e3}
    if m:
        line["reference_cpu_mtexel_s"] = float(m.group(2))
        line["reference_cpu_threads"] = int(m.group(1))
        line["reference"] = "ntc_decode --exact --bench (the reference's SSE4.1 decoder), min-time rate"
    if ref_rgb is not None:
        line["bytes_equal_to_reference"] = float(np.mean(rgb[0] == ref_rgb))
    return line


def tf32_peak_tflops(n=8192, reps=20, rounds=5):
    """cuBLAS TF32 GEMM throughput on this GPU: the best of `rounds` timings of `reps` back-to-back GEMMs (the tensor
    pipe the population kernel runs on; a secondary denominator beside the measured bf16 peak)."""
    import torch
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    a = torch.randn(n, n, device="cuda"); b = torch.randn(n, n, device="cuda"); c = torch.empty(n, n, device="cuda")
    for _ in range(3):
        torch.matmul(a, b, out=c)
    best = 0.0
    for _ in range(rounds):
        e0 = torch.cuda.Event(enable_timing=True); e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            torch.matmul(a, b, out=c)
        e1.record(); e1.synchronize()
        best = max(best, 2.0 * n ** 3 * reps / (e0.elapsed_time(e1) * 1e-3) / 1e12)
    torch.backends.cuda.matmul.allow_tf32 = prev
    return best


def tc_issued_flops_per_decode(spec) -> int:
    """Tensor FLOPs the 3xTF32 kernel issues per decode: 3 products x padded K x padded N for the two hidden
    layers (the output layer runs on the FP32 pipe)."""
    w = spec.widths
    up = lambda x, m: (x + m - 1) // m * m
    k1, n1, n2 = up(w[0] + 1, 8), up(w[1], 16), up(w[2], 16)
    return 3 * 2 * (k1 * n1 + w[1] * n2)


def pop_roofline(kernel, cfg, achieved, ffma, tf32, traffic, eval_flops, eval_avg_s, peaks):
    """The population kernel against the measured peaks. Primary: the driver-measured dense bf16 tensor peak of
    MEASURED_PEAKS.json (burst: the kernel is timed alone per launch). Secondary: the TF32 tensor pipe the kernel runs
    on (cuBLAS measured here) and the FP32 FFMA pipe (measured by the library)."""
    base = {"kernel": "k_pop_eval_tc (tcgen05 3xTF32)" if kernel == "tensor" else "k_pop_eval_x2 (packed FP32)",
            "achieved": achieved, "unit": "TFLOP/s", "traffic": traffic, "flops_per_launch": eval_flops,
            "avg_launch_ms": eval_avg_s * 1e3, "fp32_ffma_peak": ffma,
            "frac_of_fp32_ffma_peak": (achieved / ffma) if achieved else None}
    if "bf16_tflops" in peaks:
        base.update({"bound": "tensor", "peak": peaks["bf16_tflops"], "frac": (achieved / peaks["bf16_tflops"]) if achieved else None,
                     "peak_source": "of measured: MEASURED_PEAKS.json bf16_tflops (dense bf16 cuBLAS burst on this pool's B200s)"})
    else:
        base.update({"bound": "tensor", "peak": 1590.0, "frac": (achieved / 1590.0) if achieved else None,
                     "peak_source": "of fallback: 1.59 PFLOP/s dense bf16 (MEASURED_PEAKS.json absent)"})
    if kernel == "tensor" and achieved and tf32:
        issued = achieved * tc_issued_flops_per_decode(cfg.spec) / cfg.flops_per_decode()
        base.update({"tf32_peak": tf32, "frac_of_tf32_peak": achieved / tf32,
                     "tf32_peak_source": "cuBLAS TF32 GEMM (8192^3), best of 5 x 20 launches in bench.py on this GPU",
                     "issued_tensor_tflops": issued, "issued_frac_of_tf32_peak": issued / tf32,
                     "note": "achieved counts algorithmic FLOPs (2 sum n_in n_out per decode); the kernel issues "
                             f"{tc_issued_flops_per_decode(cfg.spec)} tensor FLOPs per decode (3xTF32, padded K/N)"})
    return base


def ref_cuda_leg(cfg, n1=20, span_s=24.0):
    """The reference's own CUDA backend (cuda/ntc_cuda.cu built unmodified for sm_100a, linked into the reference
    CLI as oracle/_ref/ntc_ref) on the same configuration and GPU. Runs of n1 and n2 ES iterations with no
    intermediate prints: the CLI reports the elapsed time (0.1 s resolution) at the last iteration before its final
    print, so (t(n2) - t(n1)) / (n2 - n1) is the per-iteration time without initialisation or printing. n2 is sized
    from a first 100-iteration difference so that the difference spans about span_s seconds."""
    import re
    import tempfile
    from neural_block_textures_b200 import synth
    exe = ROOT / "oracle" / "_ref" / "ntc_ref"
    if not exe.exists():
        return None
    with tempfile.TemporaryDirectory() as d:
        imgs = cfg.images()
        paths = []
        for t, im in enumerate(imgs):
            p = Path(d) / f"in{t}.png"
            synth.write_png(p, im)
            paths.append(str(p))
        flags = [f for f in cfg.cli.replace("--write-ntcb", "").split()]
        # ES phase only (the bench step): drop --mlp-fd and its value, and the iteration count
        out = []
        skip = 0
        for f in flags:
            if skip:
                skip -= 1; continue
            if f in ("--mlp-fd", "--iters"):
                skip = 1; continue
            out.append(f)

        def elapsed(n):
            r = subprocess.run([str(exe), *paths, *out, "--iters", str(n), "--print-every", "100000000", "--rng", "hash", "--cuda",
                                "--out", str(Path(d) / f"o{n}")], capture_output=True, text=True, timeout=900)
            if r.returncode != 0:
                raise RuntimeError(f"ntc_ref exited {r.returncode}: {(r.stdout + r.stderr)[-300:]}")
            m = re.findall(rf"iter\s+{n}\s.*\|\s+([0-9.]+)s \(", r.stdout)
            if not m:
                raise RuntimeError("could not parse the reference CLI's timing line")
            return float(m[-1])
        try:
            t1 = elapsed(n1)
            t2 = elapsed(n1 + 100)
            est = max((t2 - t1) / 100, 5e-4)
            n2 = n1 + max(100, int(span_s / est))
            if n2 > n1 + 100:
                t2 = elapsed(n2)
            else:
                n2 = n1 + 100
        except RuntimeError as e:
            return {"unavailable": str(e)}
    ms = 1e3 * (t2 - t1) / (n2 - n1)
    dec = sum(cfg.decodes_per_iter().values())
    return {"value": dec / (ms * 1e-3), "unit": "decodes/s", "ms_per_step": ms, "kind": "reference CUDA backend (ntc_ref, sm_100a)",
            "method": f"wall clock of the reference CLI, ({n2} - {n1}) ES iterations (0.1 s print resolution), same synthetic input"}


class Arm:
    """One configuration set up on this rank: the trainer on its own stream and, for N > 1, the sharded driver."""

    def __init__(self, cfg, args, world, rank, dist):
        import torch
        from neural_block_textures_b200 import Trainer
        from neural_block_textures_b200.shard import ShardedES, NativeShardedES, pair_range
        self.cfg, self.dist = cfg, dist
        spec = cfg.spec
        self.z0, self.p0 = spec.init_params()
        self.tr = Trainer()
        ok, why = self.tr.init(spec.model_desc(), self.z0, self.p0, cfg.target())
        if not ok:
            raise SystemExit(f"init failed: {why}")
        self.stream = torch.cuda.Stream()
        self.tr.set_stream(self.stream.cuda_stream)
        self.tr.set_pop_kernel(args.pop_kernel == "tensor")
        self.N, self.M, K = cfg.pairs, cfg.batch, cfg.lat_pairs
        p0, p1 = pair_range(self.N, world, rank)
        self.per = p1 - p0
        self.has_lat = len(spec.levels) > 1 or not spec.qat_bits
        self.qat = bool(spec.qat_bits)
        self.K = K
        self.Kl = K if self.has_lat else 0
        self.sharded = self.native = None
        L0 = spec.levels[0]
        self.dct_pull = 0.0
        if spec.dct_q:
            self._dct_live(spec)
        if world > 1 and args.shard_driver == "native":
            self.native = NativeShardedES(self.tr, dist, device="cuda",
                                          p2p=(self.N, self.Kl, self.qat) if args.exchange == "p2p" else None)
            for mode in (1, 2):
                ok, _, _, why = self.native.plan(mode, self.N, self.M, self.Kl, self.qat)
                if not ok:
                    raise SystemExit(f"native sharded iteration does not apply: {why}")
        elif world > 1:
            self.sharded = ShardedES(self.tr, dist, self.N, device="cuda", stream=self.stream, K=self.Kl, image=(spec.W, spec.H),
                                     level0=(L0.W, L0.H, L0.C) if spec.qat_bits else None, P=spec.P)

    def _dct_live(self, spec):
        """A DCT-coded level 0 (config 4) goes live as the reference trainer's switch does (main.cpp:4099-4107): scale
        codes from the sensitivity probe (here the device probe), the step tables of --dct-q, the default --dct-lambda
        recipe with truncation and the ES rate term (lambda-lo 0.25), the default dead-zone (off) and shadow pull (0.01).
        The symbols start at zero and the first latent step's snap derives them from the shadow latent."""
        from neural_block_textures_b200 import abi, dct
        tr = self.tr
        codes, _ = tr.dct_probe()
        C0 = spec.levels[0].C
        steps = np.ascontiguousarray(np.concatenate([dct.build_steps(q, spec.dct_dc_step) for q in spec.dct_q]).reshape(-1), np.int32)
        lam = dct.lambda_recipe(list(spec.dct_q))
        d = abi.DctDesc()
        d.live, d.C, d.BW, d.BH, d.N, d.dc_step = 1, C0, spec.W // 8, spec.H // 8, 8, spec.dct_dc_step
        d.rate_es, d.rate_trunc = 1, 1
        d.rate_scale = float(np.float32(lam / (16.0 * 65025.0 * spec.W * spec.H)))
        for k, v in enumerate(dct.lam_t16(lam, True)):
            d.lam_t16[k] = float(v)
        d.lo_w16, d.deadzone = 4, 0
        tr.set_dct(d, codes, np.zeros(codes.size * 64, np.int16), steps)
        self.dct_pull = 0.01
        self.dct_n0 = spec.levels[0].size

    def exchange(self) -> str:
        if self.native is None and self.sharded is None:
            return "none"
        if self.sharded is not None:
            return "torch.distributed NCCL all-gathers"
        return "peer-memory exchange kernel (CUDA IPC, NVLink)" if self.native.p2p else "NCCL in-place all-gathers"

    def step(self, it):
        c, tr = self.cfg, self.tr
        if self.native is not None:
            self.native.iteration(it, 1, c.mlp_sigma, c.mlp_lr, self.N, self.M, self.Kl, c.lat_sigma, c.lat_lr, self.qat)
        elif self.sharded is None:
            tr.mlp_step(it, c.mlp_sigma, c.mlp_lr, self.N, self.M)
            if self.has_lat:
                tr.lat_step(it, c.lat_sigma, c.lat_lr, self.K)
            if self.dct_pull > 0.0:
                tr.shadow_pull(0, self.dct_n0, self.dct_pull)
            if self.qat:
                tr.qat_search()
        else:
            self.sharded.step(it, c.mlp_sigma, c.mlp_lr, self.M)
            if self.has_lat:
                self.sharded.lat_step(it, c.lat_sigma, c.lat_lr, self.K)
            if self.qat:
                self.sharded.qat_search()

    def fd_step(self, it):
        c, tr = self.cfg, self.tr
        if self.native is not None:
            self.native.iteration(it, 2, c.fd_h, c.mlp_lr, self.N, self.M, self.Kl, c.lat_sigma, c.lat_lr, self.qat)
        elif self.sharded is None:
            tr.mlp_step_fd(it, c.fd_h, c.mlp_lr, self.M)
            if self.has_lat:
                tr.lat_step(it, c.lat_sigma, c.lat_lr, self.K)
            if self.dct_pull > 0.0:
                tr.shadow_pull(0, self.dct_n0, self.dct_pull)
            if self.qat:
                tr.qat_search()
        else:
            self.sharded.fd_step(it, c.fd_h, c.mlp_lr, self.M)
            if self.has_lat:
                self.sharded.lat_step(it, c.lat_sigma, c.lat_lr, self.K)
            if self.qat:
                self.sharded.qat_search()

    def close(self):
        if self.native is not None:
            self.native.close()
            self.native = None
        self.tr.close()


def start_together(stream, dist):
    """Drain this rank's work, then line the ranks up: after this, every rank's next launch starts within host
    jitter of the others', so no rank's first timed step absorbs a peer's late start."""
    import torch
    stream.synchronize()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
        torch.cuda.synchronize()


def max_over_ranks(vals, dist):
    """Element-wise max over ranks of a list of floats (device-side all-reduce, identical steps on every rank)."""
    if not dist:
        return list(vals)
    import torch
    t = torch.tensor(list(vals), dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.cpu()]


def timed_steps(arm, step_fn, it, steps, flush, dist):
    """`steps` iterations, each bracketed by CUDA events on the trainer's stream, the L2 flushed before each outside
    the events. Returns (per-step ms of this rank, next iteration number)."""
    import torch
    evs = []
    for _ in range(steps):
        with torch.cuda.stream(arm.stream):
            flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True); e1 = torch.cuda.Event(enable_timing=True)
            e0.record(arm.stream)
        step_fn(it); it += 1
        with torch.cuda.stream(arm.stream):
            e1.record(arm.stream)
        evs.append((e0, e1))
    arm.stream.synchronize()
    return [a.elapsed_time(b) for a, b in evs], it


def phase_breakdown(arm, step, it, nb, flush, dist):
    """Per-phase breakdown: a separate pass of nb steps with every kernel class timed (device time of this library's
    kernels and, under the native sharded driver, of the exchanges; the rest of a step is idle gaps). This rank's
    figures, ms per step."""
    import torch
    tr, stream = arm.tr, arm.stream
    tr.kernel_timing_only(None)
    tr.kernel_timing(True)
    start_together(stream, dist)
    for _ in range(nb):
        with torch.cuda.stream(stream):
            flush.zero_()
        step(it); it += 1
    stream.synchronize()
    breakdown = {}
    for cls in ("mlp_eval", "lat_eval", "qat", "batch", "noise", "mlp_finish", "mlp_grad", "lat_noise", "lat_gather", "dct_rate",
                "adam", "snap", "exchange"):
        ms_c, n_c = tr.kernel_time(cls)
        if n_c:
            breakdown[cls] = ms_c / nb
    tr.kernel_timing(False)
    return breakdown, it


def cfg5_leg(args, world, rank, dist, flush):
    """The north star's scaling configuration (config 5: 2048^2, population 32768) on the same N GPUs, same timing
    rules as the headline (warm-up, ranks lined up, L2 flushed between steps, CUDA events, max over ranks)."""
    from neural_block_textures_b200 import model
    cfg = model.config(5)
    arm = Arm(cfg, args, world, rank, dist)
    it = 1
    for _ in range(args.warmup):
        arm.step(it); it += 1
    start_together(arm.stream, dist)
    per, it = timed_steps(arm, arm.step, it, args.steps, flush, dist)
    tot, med = max_over_ranks([sum(per), statistics.median(per)], dist)
    dec = sum(cfg.decodes_per_iter().values())
    out = {"workload": cfg.name, "cli": cfg.cli, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": tot / args.steps, "ms_per_step_median": med, "value": dec * args.steps / (tot * 1e-3),
           "unit": "decodes/s", "decodes_per_step": cfg.decodes_per_iter(), "exchange": arm.exchange(),
           "scaling": "strong", "l2": "flushed between steps (256 MiB memset outside the timed events)",
           "note": "efficiency at N = value(N) / (N value(1)) over the cfg5 objects of the per-N lines"}
    nb = min(args.steps, 20)
    breakdown, it = phase_breakdown(arm, arm.step, it, nb, flush, dist)
    out["phase_ms_per_step"] = {**breakdown, "kernels_total": sum(v for k, v in breakdown.items() if k != "exchange"),
                                "note": f"rank {rank}, separate pass of {nb} steps with every kernel class timed"}
    arm.close()
    return out


def main():
    args = parse()
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        reference_arm(args, world, rank)
        return
    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    from neural_block_textures_b200 import load_library, model

    cfg = model.config(args.config)
    spec = cfg.spec
    arm = Arm(cfg, args, world, rank, dist)
    tr, stream = arm.tr, arm.stream
    N, M = arm.N, arm.M
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    dec = cfg.decodes_per_iter()
    decodes = sum(dec.values())
    step, fd_step = arm.step, arm.fd_step

    it = 1
    for _ in range(args.warmup):
        step(it); it += 1
    start_together(stream, dist)
    # Inside the timed region only the population kernel carries CUDA events (the roofline's launch time): events
    # around every launch cost host calls that, on several GPUs, can outlast the device work of a step.
    tr.kernel_timing(True)
    tr.kernel_timing_only("mlp_eval")
    launches0 = tr.launch_count()
    with ClockSampler(local) as clk:
        time.sleep(0.6)            # nvidia-smi's first sample lands before the timed steps start
        start_together(stream, dist)
        per_step, it = timed_steps(arm, step, it, args.steps, flush, dist)
    torch.cuda.synchronize()
    launches = tr.launch_count() - launches0
    eval_ms, eval_n = tr.kernel_time("mlp_eval")
    tr.kernel_timing(False)
    ms, ms_med, ms_first = max_over_ranks([sum(per_step), statistics.median(per_step), per_step[0]], dist)

    nb = min(args.steps, 100)
    breakdown, it = phase_breakdown(arm, step, it, nb, flush, dist)
    value = decodes * args.steps / (ms * 1e-3)

    # ---- FD-phase iterations (mlp_step_fd + lat_step + qat_search), same timing rules
    fd_line = None
    if args.fd_steps > 0:
        for _ in range(3):
            fd_step(it); it += 1
        start_together(stream, dist)
        fper, it = timed_steps(arm, fd_step, it, args.fd_steps, flush, dist)
        fms, fmed = max_over_ranks([sum(fper), statistics.median(fper)], dist)
        fdec = cfg.decodes_per_iter(fd=True)
        fd_line = {"steps": args.fd_steps, "ms_per_step": fms / args.fd_steps, "ms_per_step_median": fmed, "decodes_per_step": fdec,
                   "value": sum(fdec.values()) * args.fd_steps / (fms * 1e-3), "unit": "decodes/s",
                   "kernel": ("k_pop_eval_tc (tcgen05 3xTF32)" if tr.pop_kernel() == "tensor" else "k_pop_eval_x2 (packed FP32, exact)")
                             + ": the stats pair and the 2P FD candidates in one launch"}

    # ---- end to end through the public API with host buffers (pinned), copies inside the timed region
    zh = torch.empty(spec.nz, dtype=torch.float32, pin_memory=True).numpy()
    ph = torch.empty(spec.P, dtype=torch.float32, pin_memory=True).numpy()
    zh[:] = arm.z0; ph[:] = arm.p0
    zo = torch.empty(spec.nz, dtype=torch.float32, pin_memory=True).numpy()   # the step's results, read into pinned memory
    po = torch.empty(spec.P, dtype=torch.float32, pin_memory=True).numpy()
    e2e_steps = args.e2e_steps
    for _ in range(2):
        tr.upload_model(zh, ph); step(it); it += 1
        tr.download_model(zo, po); tr.mlp_stats()
    start_together(stream, dist)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        tr.upload_model(zh, ph)
        step(it); it += 1
        tr.download_model(zo, po)
        tr.mlp_stats()
    e2e_s = max_over_ranks([time.perf_counter() - t0], dist)[0]
    e2e_value = decodes * e2e_steps / e2e_s
    h2d = 4 * (spec.nz + spec.P)
    d2h = 4 * (spec.nz + spec.P) + 16 * N
    kernel = tr.pop_kernel()
    pprint = progress_print_leg(tr, cfg, not args.no_cpu_baseline) if (rank == 0 and world == 1) else None
    exchange = arm.exchange()
    # ---- the same ES iterations with NCCL all-gathers in place of the peer-memory exchange (N > 1, native driver): the
    # north star's fitness exchange by NCCL, timed by the same rules for comparison (the peer exchange is released on
    # every rank first; the library then issues the in-place NCCL all-gathers on its own communicator)
    nccl_line = None
    if arm.native is not None and arm.native.p2p:
        tr.p2p_release()
        dist.barrier()
        arm.native.p2p = False
        for _ in range(3):
            step(it); it += 1
        start_together(stream, dist)
        nper, it = timed_steps(arm, step, it, args.steps, flush, dist)
        nms, nmed = max_over_ranks([sum(nper), statistics.median(nper)], dist)
        nccl_line = {"exchange": "NCCL in-place all-gathers (library communicator)", "steps": args.steps,
                     "ms_per_step": nms / args.steps, "ms_per_step_median": nmed,
                     "value": decodes * args.steps / (nms * 1e-3), "unit": "decodes/s"}

    arm.close()

    # ---- the north star's scaling configuration on the same GPUs (every rank takes part)
    cfg5 = cfg5_leg(args, world, rank, dist, flush) if not args.no_cfg5 else None

    if rank == 0:
        lib = load_library()
        ffma = float(lib.ntcb_fp32_peak_tflops())
        tf32 = tf32_peak_tflops() if kernel == "tensor" else None
        fpd = cfg.flops_per_decode()
        eval_flops = 2 * arm.per * M * fpd if world > 1 else 2 * N * M * fpd
        eval_avg_s = (eval_ms / max(eval_n, 1)) * 1e-3
        achieved = eval_flops / eval_avg_s / 1e12 if eval_n else None
        peaks = {}
        pk = ROOT / "MEASURED_PEAKS.json"
        if pk.exists():
            peaks = json.loads(pk.read_text())
        traffic = None
        tf = ROOT / "profiles" / "traffic.json"
        if tf.exists():
            traffic = json.loads(tf.read_text()).get(cfg.name, {}).get("mlp_eval_dram_bytes_per_launch")
        line = {
            "metric": "candidate-pixel decodes/s (ES training iteration)", "value": value, "unit": "decodes/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "ms_per_step_median": ms_med, "ms_first_step": ms_first,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": cfg.name, "cli": cfg.cli, "decodes_per_step": dec, "parallelism": f"population x{world}",
                       "exchange": exchange, "pop_kernel": kernel,
                       "l2": "flushed between steps (256 MiB memset outside the timed events)"},
            "roofline": pop_roofline(kernel, cfg, achieved, ffma, tf32, traffic, eval_flops, eval_avg_s, peaks),
            "phase_ms_per_step": {**breakdown, "kernels_total": sum(v for k, v in breakdown.items() if k != "exchange"),
                                  "note": f"separate pass of {nb} steps with every kernel class timed (events around each launch)"},
            "e2e": {"value": e2e_value, "unit": "decodes/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "Trainer.upload_model (pinned host) + mlp_step + lat_step + qat_search + download_model (into pinned host arrays) + mlp_stats"},
            "gpu_launches": launches,
            "fd_phase": fd_line,
            "nccl_exchange": nccl_line,
            "cfg5": cfg5,
            "clocks": clk.summary(),
        }
        if pprint is not None:
            line["progress_print"] = pprint
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_leg(cfg)
            line["ntcb_decode"] = ntcb_decode_leg()
        if world == 1 and not args.no_ref_cuda:
            line["ref_cuda_backend"] = ref_cuda_leg(cfg)
        print(json.dumps(line))
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
