#!/usr/bin/env python3
"""Throughput of the exact-integer SD-turbo UNet step on B200s: UNet inferences/s, batch 8 x 2 lanes per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl vela|reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N ...

A step is one UNet denoising step (noise -> UNet -> x0) on every lane of every GPU: 2 lanes x batch 8 =
16 inferences per GPU.  Inferences are independent; each GPU (one process each) runs its own model copy on
a disjoint block of seeds with no collective on the data path ("scaling": "weak").

Our arm (--impl vela), one JSON line from rank 0:
  value       device-timed: the step graphs replayed on device-resident seeds (vela_engine_launch_device),
              both lanes' streams bracketed by CUDA events; K steps; max over ranks.
  e2e         the public API a user calls (Engine.submit / Engine.collect from one host thread per lane,
              the reference's runBench pattern, src/main.cpp:111-162): host seeds in, host x0 out, the H2D and
              D2H copies inside the timed region; wall clock between synchronised barriers, max over ranks.
  roofline    the dominant kernel of the step (exact attention at the largest self-attention shape,
              8 x 5 heads x 4096 tokens x 64), timed live with CUDA events on the stream it is launched on.
  cpu_baseline the CPU restatement of the integer spec (oracle/, OpenMP over the host cores), one bounded
              sample: one step at batch 1 (rank 0, N = 1 only).
  x0 check    the golden seeds of the reference engine's fixture must give the reference engine's x0 bytes,
              and every rank must produce the same x0 for the same seeds.

The reference arm (--impl reference) runs the reference engine itself, compiled from the reference's own
sources (oracle/_ref/libvela_ref.so, built by `make -C oracle ref`), through its own Engine::submit /
collect with one host thread per lane, on the same model bytes, batch, lanes and steps.  Its process loads no
library of the product: the model file comes from the test side's writer (oracle/synth_model.c), which gives the
same bytes as vela_synth_model_write.  Its cpu_baseline is the oracle's CPU restatement (the reference has no CPU
implementation of the path), the same bounded sample as our arm's.
"""
import argparse
import hashlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROMPT = [320, 736, 3240]
MODEL_SEED = 1
METRIC = "UNet inferences/s (SD-turbo step, batch 8 x 2 lanes per GPU, bit-exact x0)"
UNIT = "inferences/s"
# algorithmic int8 work of one self-attention launch at 8 x 5 heads x 4096 x 4096 x 64: QK^T and PV,
# each a 16-bit x 16-bit product carried as 4 int8 planes -> 2 * 4 * 8*5*4096*4096*64 MACs, 2 ops per MAC
ATTN_SHAPE = dict(B=8, heads=5, T=4096)
ATTN_OPS = 2 * 4 * 2 * 8 * 5 * 4096 * 4096 * 64
ATTN_PROFILE = os.path.join(ROOT, "profiles", "attention_self_b8h5t4096.md")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["vela", "reference"], default="vela")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--lanes", type=int, default=2)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-roofline", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel", choices=["attention", "gemm", "gn_conv", "linear", "geglu", "qkv", "norms"], default=None,
                    help="run only the named kernel(s) at the BASELINE config shape (attention: config 2, gemm: config 1, "
                         "gn_conv: config 3 at 320 ch 64x64, or --conv-level 1 / 2 / 3 for 640 ch 32x32 / 1280 ch 16x16 / 1280 ch 8x8), "
                         "linear: the UNet's int32-input linear with residual at 64x64 (M 32768, K --linear-k, N 320), "
                         "geglu: its planar GEGLU GEMM (M 32768, K 320, N 2560); qkv: the merged q|k|v GEMM with head "
                         "quantisation (M 32768, K 320, N 960); norms: GroupNorm statistics, "
                         "GroupNorm+SiLU apply and LayerNorm->planes at 320 ch 64x64, each timed alone; "
                         "print their CUDA-event times as one JSON line and exit; with --impl reference the reference's own "
                         "kernels at the same shapes")
    ap.add_argument("--linear-k", type=int, default=320)
    ap.add_argument("--conv-level", type=int, default=0, choices=[0, 1, 2, 3])
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)
    return a


# ------------------------------------------------------------------ process group / devices
class Ranks:
    def __init__(self):
        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = False

    def init(self):
        import torch
        torch.cuda.set_device(self.local)
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            # NCCL's own messages (its version banner when NCCL_DEBUG is set) go to a per-rank file in the temp
            # directory, not to stdout, which carries only the bench's JSON line
            os.environ.setdefault("NCCL_DEBUG_FILE", os.path.join(tempfile.gettempdir(), f"vela_bench_nccl.{self.rank}.log"))
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local))
            self.pg = True

    def barrier(self):
        if self.pg:
            import torch.distributed as dist
            dist.barrier()

    def max(self, v):
        from vela_b200.dist import max_over_ranks
        import torch
        return max_over_ranks(v, torch.device("cuda", self.local)) if self.pg else float(v)

    def agree(self, digest):
        from vela_b200.dist import digests_agree
        import torch
        return digests_agree(digest, torch.device("cuda", self.local)) if self.pg else True

    def close(self):
        if self.pg:
            import torch.distributed as dist
            dist.destroy_process_group()


class Clocks:
    """nvidia-smi samples every 200 ms while running (the GPU's clocks and throttle reasons)"""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu, self.p, self.f = gpu, None, None

    def __enter__(self):
        try:
            self.f = tempfile.TemporaryFile("w+")
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.Q, "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        return self

    def __exit__(self, *exc):
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(5)
            except subprocess.TimeoutExpired:
                self.p.kill()

    def summary(self):
        if not self.p:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.f.seek(0)
        rows = [[c.strip() for c in line.split(",")] for line in self.f if line.count(",") >= 7]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        sm, reasons, smax, power = [], set(), None, []
        for r in rows:
            try:
                sm.append(float(r[1])); smax = float(r[2]); power.append(float(r[3]))
            except ValueError:
                continue
            for i, n in enumerate(names):
                if r[4 + i].lower() == "active":
                    reasons.add(n)
        load = [s for s, p in zip(sm, power) if p > 300] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


def model_file(R, writer):
    """The seeded synthetic model (~1.2 GB), written once per box and arm: rank 0 writes it to a temporary name and
    renames it into place, the other ranks wait at a barrier, so N ranks share one file.  `writer` is "product"
    (vela_synth_model_write, our arm) or "oracle" (the test side's writer, the reference arm, whose process must not
    load the product library); both give the same bytes for the same seed (tests/test_synth_model_cpu.py)."""
    path = os.path.join(tempfile.gettempdir(), f"vela_synth_seed{MODEL_SEED}_{writer}.poisd")
    if R.rank == 0 and not (os.path.exists(path) and os.path.getsize(path) > (1 << 30)):
        tmp = f"{path}.tmp{os.getpid()}"
        if writer == "product":
            import vela_b200 as V
            V.synth_model_write(tmp, MODEL_SEED)
        else:
            from oracle import pyoracle as O
            O.synth_model_write(tmp, MODEL_SEED)
        os.replace(tmp, path)
    R.barrier()
    return path


def loaded_native_libs():
    """shared libraries of this repository mapped into this process (from /proc/self/maps)"""
    out = set()
    try:
        with open("/proc/self/maps") as f:
            for line in f:
                p = line.split()[-1] if line.strip() else ""
                if p.endswith(".so") and p.startswith(ROOT):
                    out.add(os.path.relpath(p, ROOT))
    except OSError:
        pass
    return sorted(out)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def profile_traffic():
    """DRAM bytes per launch of the roofline kernel, from the committed ncu summary (None if not captured yet)"""
    try:
        with open(ATTN_PROFILE) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return int(line.split(":")[1].split()[0])
    except (OSError, ValueError):
        pass
    return None


# ------------------------------------------------------------------ the dominant kernel, live
class AttentionCase:
    """Quantised operands of one self-attention at 8 x 5 heads x 4096 x 64 (activations uniform over the int16
    range, seeded), built by the library's own quantisers; launch() runs vela_fused_attention once."""

    def __init__(self, device):
        import torch
        import vela_b200 as V
        self.t, self.V, self.L = torch, V, V.lib()
        B, heads, T = ATTN_SHAPE["B"], ATTN_SHAPE["heads"], ATTN_SHAPE["T"]
        C, G, Tp = 64 * heads, B * heads, (T + 127) // 128 * 128
        g = torch.Generator(device=device); g.manual_seed(2)
        d = lambda *s, dt: torch.zeros(s, dtype=dt, device=device)
        X = [torch.randint(-32768, 32768, (B, T, C), generator=g, device=device, dtype=torch.int32) for _ in range(3)]
        self.q = [d(G, Tp, 64, dt=torch.int8), d(G, Tp, 64, dt=torch.int8), d(G, Tp, dt=torch.int32)] + [d(G, Tp, dt=torch.int64) for _ in range(3)]
        self.k = [d(G, Tp, 64, dt=torch.int8), d(G, Tp, 64, dt=torch.int8), d(G, Tp, dt=torch.int32)] + [d(G, Tp, dt=torch.int64) for _ in range(3)]
        self.v = [d(G, 64, Tp, dt=torch.int8), d(G, 64, Tp, dt=torch.int8), d(G, 64, dt=torch.int32), d(G, 64, dt=torch.int64)]
        colmax = d(G, 64, dt=torch.int32)
        self.lexp = torch.from_numpy(np.rint(1073741824.0 * np.exp(-np.arange(1025) / 64.0)).astype(np.int32)).to(device)
        self.out = d(B, T, C, dt=torch.int32); self.rm = d(B * T, dt=torch.int32)
        self.stream = torch.cuda.current_stream(device)
        P = lambda x: x.data_ptr()
        st = self.stream.cuda_stream
        V.check(self.L.vela_quant_heads(st, P(X[0]), B, T, C, heads, Tp, *[P(x) for x in self.q]))
        V.check(self.L.vela_quant_heads(st, P(X[1]), B, T, C, heads, Tp, *[P(x) for x in self.k]))
        V.check(self.L.vela_quant_v(st, P(X[2]), B, T, C, heads, Tp, *[P(x) for x in self.v], P(colmax)))
        self.args = (P(self.q[0]), P(self.q[1]), P(self.q[2]), P(self.q[3]), P(self.q[4]), P(self.k[0]), P(self.k[1]), P(self.k[2]),
                     P(self.k[5]), P(self.v[0]), P(self.v[1]), P(self.v[2]), P(self.v[3]), B, heads, T, Tp, T, Tp, 0,
                     P(self.lexp), C, None, None, P(self.out), P(self.rm))
        del X
        torch.cuda.synchronize(device)

    def launch(self):
        self.V.check(self.L.vela_fused_attention(self.stream.cuda_stream, *self.args))

    def time_ms(self, warmup=3, iters=10):
        torch = self.t
        for _ in range(warmup):
            self.launch()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(self.stream)
        for _ in range(iters):
            self.launch()
        e1.record(self.stream)
        e1.synchronize()
        assert self.L.vela_device_error(1) == 0, "attention kernel reported a device error"
        return e0.elapsed_time(e1) / iters


def _time_ms(stream, fn, warmup=3, iters=10):
    import torch
    for _ in range(warmup):
        fn()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(iters):
        fn()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / iters


class GemmCase:
    """Config 1: planar A (hi/lo of int16 uniform over [-32768, 32767]) M 4096 x K 320, W int8 320 x 320, e in [0, 12)."""

    def __init__(self, device):
        import ctypes
        import torch
        import vela_b200 as V
        from vela_b200 import abi
        self.t, self.V, self.L = torch, V, V.lib()
        M, N, K = 4096, 320, 320
        g = torch.Generator(device=device); g.manual_seed(1)
        q = torch.randint(-32768, 32768, (M, K), generator=g, device=device, dtype=torch.int32)
        self.hi = (q >> 8).to(torch.int8); self.lo = ((q & 255) - 128).to(torch.int8)
        self.W = torch.randint(-127, 128, (N, K), generator=g, device=device, dtype=torch.int32).to(torch.int8)
        cst = torch.zeros((N, 4), dtype=torch.int32, device=device)
        cst[:, 0] = torch.randint(16384, 32768, (N,), generator=g, device=device, dtype=torch.int32)
        cst[:, 1] = torch.randint(20, 30, (N,), generator=g, device=device, dtype=torch.int32)
        cst[:, 2] = torch.randint(-50000, 50000, (N,), generator=g, device=device, dtype=torch.int32)
        cst[:, 3] = self.W.to(torch.int32).sum(1)
        self.cst = cst
        self.e = torch.randint(0, 12, (M,), generator=g, device=device, dtype=torch.int32)
        self.Y = torch.empty((M, N), dtype=torch.int32, device=device)
        a = abi.ASrc(); a.src = abi.SRC_I8; a.hi = self.hi.data_ptr(); a.lo = self.lo.data_ptr(); a.ld8 = K; a.e = self.e.data_ptr()
        E = abi.AEpi(); E.epi = abi.EPI_PLAIN; E.Y = self.Y.data_ptr(); E.ldy = N
        self.a, self.E, self.shape = a, E, (M, N, K)
        self.stream = torch.cuda.current_stream(device)
        self.ptr = ctypes.c_void_p
        self.byref = ctypes.byref

    def launch(self):
        M, N, K = self.shape
        self.V.check(self.L.vela_gemm_w8a16(self.stream.cuda_stream, self.byref(self.a), M, M, self.ptr(self.W.data_ptr()), K, N, N, K,
                                            self.ptr(self.cst.data_ptr()), self.byref(self.E)))

    def report(self):
        M, N, K = self.shape
        ms = _time_ms(self.stream, self.launch)
        ops = 2 * 2 * M * N * K
        byt = M * K * 2 + N * K + M * 4 + M * N * 4
        return {"kernel": "gemm_w8a16 planar (config 1)", "M": M, "N": N, "K": K, "ms": round(ms, 4),
                "int8_tops": round(ops / ms / 1e9, 2), "gbs": round(byt / ms / 1e6, 1)}


class GnConvCase:
    """Config 3: GroupNorm (32 groups) + SiLU of int32 NHWC [8, H*W, C] (uniform over the int16 range), pixel max,
    then the 3x3 conv C -> C with int8 weights the way the engine runs it, given the engine's 64 MiB split-K
    workspace: at 320 channels (64x64) the implicit conv (3x3 window exponents, windows quantised on load); at 640
    and 1280 channels (32x32 and below) the explicit im2col into hi / lo planes (window exponents included) and the
    planar GEMM.
    Levels 0-2 are the configuration's shapes; level 3 (1280 ch at 8x8, the UNet's deepest level) is the shape where
    the GEMM splits K and runs the split-K reduction.  The implicit form is also timed at every level."""
    LEVELS = [(64, 320), (32, 640), (16, 1280), (8, 1280)]

    def __init__(self, device, level):
        import ctypes
        import torch
        import vela_b200 as V
        from vela_b200 import abi
        self.t, self.V, self.L = torch, V, V.lib()
        Hh, C = self.LEVELS[level]
        B, T, N, K = 8, Hh * Hh, C, 9 * C
        g = torch.Generator(device=device); g.manual_seed(3)
        ri = lambda lo, hi, shape: torch.randint(lo, hi, shape, generator=g, device=device, dtype=torch.int32)
        self.X = ri(-32768, 32768, (B, T, C))
        self.gam = ri(65536 - 16384, 65536 + 16384, (C,)); self.beta = ri(-8192, 8192, (C,))
        xs = np.arange(2049, dtype=np.float64) / 64.0 - 16.0
        self.Lsig = torch.from_numpy(np.rint(65536.0 / (1.0 + np.exp(-xs))).astype(np.int32)).to(device)
        self.gs = torch.zeros((B * 32, 6), dtype=torch.int64, device=device)
        self.Y = torch.empty((B, T, C), dtype=torch.int32, device=device)
        self.pm = torch.empty((B * T,), dtype=torch.int32, device=device)
        self.ce = torch.empty((B * T,), dtype=torch.int32, device=device)
        self.W = ri(-127, 128, (N, K)).to(torch.int8)
        cst = torch.zeros((N, 4), dtype=torch.int32, device=device)
        cst[:, 0] = ri(16384, 32768, (N,)); cst[:, 1] = ri(20, 30, (N,)); cst[:, 2] = ri(-50000, 50000, (N,)); cst[:, 3] = self.W.to(torch.int32).sum(1)
        self.cst = cst
        self.out = torch.empty((B, T, N), dtype=torch.int32, device=device)
        a = abi.ASrc(); a.src = abi.SRC_CONV32; a.img = self.Y.data_ptr(); a.H = Hh; a.W = Hh; a.C = C; a.stride = 1; a.Ho = Hh; a.Wo = Hh
        a.K = K; a.e = self.ce.data_ptr()
        self.ws = torch.empty((64 << 20,), dtype=torch.uint8, device=device)
        E = abi.AEpi(); E.epi = abi.EPI_PLAIN; E.Y = self.out.data_ptr(); E.ldy = N
        E.workspace = self.ws.data_ptr(); E.workspace_bytes = 64 << 20
        self.a, self.E, self.dims = a, E, (B, Hh, C, T, N, K)
        # the engine's rule (explicit_im2col in engine.cu): 640 or more output channels on at most 32 x 32 pixels
        self.explicit = N >= 640 and T <= 1024
        if self.explicit:
            Mp = (B * T + 63) // 64 * 64
            self.hi = torch.empty((Mp, K), dtype=torch.int8, device=device); self.lo = torch.empty_like(self.hi)
            self.pe = torch.empty((Mp,), dtype=torch.int32, device=device)
            ap = abi.ASrc(); ap.src = abi.SRC_I8; ap.hi = self.hi.data_ptr(); ap.lo = self.lo.data_ptr(); ap.ld8 = K
            ap.e = self.pe.data_ptr(); ap.K = K
            self.ap, self.Mp = ap, Mp
        self.stream = torch.cuda.current_stream(device)
        self.P = lambda x: ctypes.c_void_p(x.data_ptr())
        self.byref = ctypes.byref

    def gn(self):
        B, Hh, C, T, N, K = self.dims
        st, P = self.stream.cuda_stream, self.P
        self.V.check(self.L.vela_gn_stats(st, P(self.X), B, T, C, 32, 100000, P(self.gs)))
        self.V.check(self.L.vela_gn_apply_row(st, P(self.X), B, T, C, 32, P(self.gs), P(self.gam), P(self.beta), P(self.Lsig),
                                              P(self.Y), P(self.pm), None, None, None, 0))

    def conv_implicit(self):
        B, Hh, C, T, N, K = self.dims
        st, P = self.stream.cuda_stream, self.P
        self.V.check(self.L.vela_conv_e(st, P(self.pm), B, Hh, Hh, 1, P(self.ce)))
        self.V.check(self.L.vela_gemm_w8a16(st, self.byref(self.a), B * T, B * T, P(self.W), K, N, N, K, P(self.cst), self.byref(self.E)))

    def conv(self):
        if not self.explicit:
            return self.conv_implicit()
        B, Hh, C, T, N, K = self.dims
        st, P = self.stream.cuda_stream, self.P
        self.V.check(self.L.vela_im2col3(st, P(self.Y), P(self.pm), B, Hh, Hh, C, 1, P(self.hi), P(self.lo), P(self.pe), K))
        self.V.check(self.L.vela_gemm_w8a16(st, self.byref(self.ap), self.Mp, B * T, P(self.W), K, N, N, K, P(self.cst), self.byref(self.E)))

    def launch(self):
        self.gn(); self.conv()

    def report_norms(self):
        """GroupNorm statistics, GroupNorm + SiLU apply (int32 + pixel max), GroupNorm -> int8 planes (the transformer
        blocks' input norm) and LayerNorm -> planes, timed apart"""
        import torch
        B, Hh, C, T, N, K = self.dims
        st, P = self.stream.cuda_stream, self.P
        stats = lambda: self.V.check(self.L.vela_gn_stats(st, P(self.X), B, T, C, 32, 100000, P(self.gs)))
        apply = lambda: self.V.check(self.L.vela_gn_apply_row(st, P(self.X), B, T, C, 32, P(self.gs), P(self.gam), P(self.beta), P(self.Lsig),
                                                               P(self.Y), P(self.pm), None, None, None, 0))
        stats()
        hi = torch.empty((B * T, C), dtype=torch.int8, device=self.X.device); lo = torch.empty_like(hi)
        e = torch.empty((B * T,), dtype=torch.int32, device=self.X.device)
        ln = lambda: self.V.check(self.L.vela_lnorm_q(st, P(self.X), B * T, C, P(self.gam), P(self.beta), 100000, P(hi), P(lo), P(e), C))
        applyq = lambda: self.V.check(self.L.vela_gn_apply_row(st, P(self.X), B, T, C, 32, P(self.gs), P(self.gam), P(self.beta), None,
                                                                None, None, P(hi), P(lo), P(e), C))
        ts, ta, tl = _time_ms(self.stream, stats), _time_ms(self.stream, apply), _time_ms(self.stream, ln)
        tq = _time_ms(self.stream, applyq)
        nb = B * T * C * 4
        return {"kernel": "norms (320 ch 64x64)", "gn_stats_ms": round(ts, 4), "gn_stats_gbs": round(2 * nb / ts / 1e6, 1),
                "gn_apply_ms": round(ta, 4), "gn_apply_gbs": round((2 * nb + B * T * 4) / ta / 1e6, 1),
                "gn_apply_q_ms": round(tq, 4), "gn_apply_q_gbs": round((nb + nb // 2 + B * T * 4) / tq / 1e6, 1),
                "lnorm_q_ms": round(tl, 4), "lnorm_q_gbs": round((nb + nb // 2) / tl / 1e6, 1)}

    def report(self):
        B, Hh, C, T, N, K = self.dims
        self.gn()
        gms, cms, ims = _time_ms(self.stream, self.gn), _time_ms(self.stream, self.conv), _time_ms(self.stream, self.conv_implicit)
        ops = 2 * 2 * B * T * N * K
        return {"kernel": "GroupNorm+SiLU -> 3x3 conv (config 3)", "B": B, "HW": Hh, "C": C,
                "gn_ms": round(gms, 4), "gn_gbs": round(B * T * C * 8 / gms / 1e6, 1),
                "conv_path": "explicit im2col + planar GEMM" if self.explicit else "implicit",
                "conv_ms": round(cms, 4), "conv_int8_tops": round(ops / cms / 1e9, 2), "implicit_conv_ms": round(ims, 4)}


class LinearCase:
    """The UNet's linears at the 64x64 level: int32 activations [32768, K] quantised on load (row max given),
    N 320, plain epilogue with residual and row max (proj_out / to_out: K 320; ff.net.2: K 1280); or the GEGLU
    GEMM on LayerNorm planes (K 320, N 2 x 1280 interleaved a|g)."""

    def __init__(self, device, kind, K):
        import ctypes
        import torch
        import vela_b200 as V
        from vela_b200 import abi
        self.t, self.V, self.L = torch, V, V.lib()
        M = 32768
        N = {"geglu": 2560, "qkv": 960}.get(kind, 320)
        g = torch.Generator(device=device); g.manual_seed(4)
        ri = lambda lo, hi, shape: torch.randint(lo, hi, shape, generator=g, device=device, dtype=torch.int32)
        self.W = ri(-127, 128, (N, K)).to(torch.int8)
        cst = torch.zeros((N, 4), dtype=torch.int32, device=device)
        cst[:, 0] = ri(16384, 32768, (N,)); cst[:, 1] = ri(20, 30, (N,)); cst[:, 2] = ri(-50000, 50000, (N,)); cst[:, 3] = self.W.to(torch.int32).sum(1)
        self.cst = cst
        self.rm_out = torch.zeros((M,), dtype=torch.int32, device=device)
        a = abi.ASrc(); E = abi.AEpi()
        if kind == "qkv":
            q = ri(-32768, 32768, (M, K))
            self.hi = (q >> 8).to(torch.int8); self.lo = ((q & 255) - 128).to(torch.int8); self.e = ri(0, 6, (M,))
            a.src = abi.SRC_I8; a.hi = self.hi.data_ptr(); a.lo = self.lo.data_ptr(); a.ld8 = K; a.e = self.e.data_ptr()
            heads, T, C = 5, 4096, 320
            G = (M // T) * heads
            z = lambda *s_, dt: torch.zeros(s_, dtype=dt, device=device)
            self.qb = [z(G, T, 64, dt=torch.int8), z(G, T, 64, dt=torch.int8), z(G, T, dt=torch.int32)] + [z(G, T, dt=torch.int64) for _ in range(3)]
            self.kb = [z(G, T, 64, dt=torch.int8), z(G, T, 64, dt=torch.int8), z(G, T, dt=torch.int32)] + [z(G, T, dt=torch.int64) for _ in range(3)]
            self.Y = z(M, C, dt=torch.int32)
            E.epi = abi.EPI_QKV; E.Y2 = self.Y.data_ptr(); E.heads = heads; E.T = T; E.TpQ = T; E.TpK = T; E.C = C
            E.qhi, E.qlo, E.qe, E.qhs, E.qls, E.qts = [x.data_ptr() for x in self.qb]
            E.khi, E.klo, E.ke, E.khs, E.kls, E.kts = [x.data_ptr() for x in self.kb]
        elif kind == "geglu":
            q = ri(-32768, 32768, (M, K))
            self.hi = (q >> 8).to(torch.int8); self.lo = ((q & 255) - 128).to(torch.int8); self.e = ri(0, 6, (M,))
            a.src = abi.SRC_I8; a.hi = self.hi.data_ptr(); a.lo = self.lo.data_ptr(); a.ld8 = K; a.e = self.e.data_ptr()
            xs = np.arange(2049, dtype=np.float64) / 64.0 - 16.0
            from math import erf, sqrt
            self.Lphi = torch.from_numpy(np.rint([65536.0 * 0.5 * (1 + erf(x / sqrt(2))) for x in xs]).astype(np.int32)).to(device)
            self.Y = torch.empty((M, N // 2), dtype=torch.int32, device=device)
            E.epi = abi.EPI_GEGLU; E.Y = self.Y.data_ptr(); E.ldy = N // 2; E.Lphi = self.Lphi.data_ptr(); E.rowmax = self.rm_out.data_ptr()
        else:
            self.X = ri(-(1 << 20), 1 << 20, (M, K))
            self.rm_in = self.X.abs().amax(1).to(torch.int32)
            self.R = ri(-(1 << 20), 1 << 20, (M, N))
            self.Y = torch.empty((M, N), dtype=torch.int32, device=device)
            a.src = abi.SRC_X32; a.x = self.X.data_ptr(); a.ldx = K; a.K = K; a.rowmax = self.rm_in.data_ptr()
            E.epi = abi.EPI_PLAIN; E.Y = self.Y.data_ptr(); E.ldy = N; E.residual = self.R.data_ptr(); E.rowmax = self.rm_out.data_ptr()
        self.a, self.E, self.shape, self.kind = a, E, (M, N, K), kind
        self.stream = torch.cuda.current_stream(device)
        self.ptr = ctypes.c_void_p
        self.byref = ctypes.byref

    def launch(self):
        M, N, K = self.shape
        self.V.check(self.L.vela_gemm_w8a16(self.stream.cuda_stream, self.byref(self.a), M, M, self.ptr(self.W.data_ptr()), K, N, N, K,
                                            self.ptr(self.cst.data_ptr()), self.byref(self.E)))

    def report(self):
        M, N, K = self.shape
        ms = _time_ms(self.stream, self.launch)
        rep = {"kernel": f"gemm_w8a16 {self.kind} (64x64 level)", "M": M, "N": N, "K": K, "ms": round(ms, 4),
               "int8_tops": round(2 * 2 * M * N * K / ms / 1e9, 2)}
        if self.kind == "linear":
            # the same product the way the engine runs it at these sizes: the input quantised once into planes with its
            # row maxima already known (vela_quant_rows_rm), then the planar GEMM
            import torch
            from vela_b200 import abi
            hi = torch.empty((M, K), dtype=torch.int8, device=self.X.device); lo = torch.empty_like(hi)
            e = torch.empty((M,), dtype=torch.int32, device=self.X.device)
            a = abi.ASrc(); a.src = abi.SRC_I8; a.hi = hi.data_ptr(); a.lo = lo.data_ptr(); a.ld8 = K; a.e = e.data_ptr()
            st = self.stream.cuda_stream
            quant = lambda: self.V.check(self.L.vela_quant_rows_rm(st, self.ptr(self.X.data_ptr()), self.ptr(self.rm_in.data_ptr()), M, K, K,
                                                                   self.ptr(hi.data_ptr()), self.ptr(lo.data_ptr()), self.ptr(e.data_ptr()), K, M))
            gemm = lambda: self.V.check(self.L.vela_gemm_w8a16(st, self.byref(a), M, M, self.ptr(self.W.data_ptr()), K, N, N, K,
                                                               self.ptr(self.cst.data_ptr()), self.byref(self.E)))
            quant()
            rep["planar_quant_ms"] = round(_time_ms(self.stream, quant), 4)
            rep["planar_gemm_ms"] = round(_time_ms(self.stream, gemm), 4)
        return rep


# ------------------------------------------------------------------ the reference's kernels at the config shapes
class RefKernels:
    """The reference's own kernels (oracle/_ref/libvela_ref.so: src/kernels.cu, gemm_hl.cu, attn.cu, gemm.cu compiled
    from its sources) timed with CUDA events at the same shapes and value distributions as our --kernel cases.
    Inputs are quantised by the reference's own quantisers, so this process loads no library of the product."""

    def __init__(self, device):
        import ctypes
        import torch
        so = os.path.join(ROOT, "oracle", "_ref", "libvela_ref.so")
        if not os.path.exists(so):
            raise FileNotFoundError(so)
        self.L = ctypes.CDLL(so)
        self.L.ref_last_error.restype = ctypes.c_char_p
        self.L.ref_set_sync.argtypes = [ctypes.c_int]
        self.t, self.dev, self.c = torch, device, ctypes
        self.L.ref_set_sync(0)

    def P(self, x):
        return self.c.c_void_p(x.data_ptr()) if x is not None else None

    def ok(self, rc):
        if rc != 0:
            raise RuntimeError("reference kernel: " + self.L.ref_last_error().decode())

    def time(self, fn, warmup=3, iters=10):
        torch = self.t
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s = torch.cuda.default_stream(self.dev)        # the harness launches on the legacy default stream
        e0.record(s)
        for _ in range(iters):
            fn()
        e1.record(s)
        e1.synchronize()
        return e0.elapsed_time(e1) / iters

    def ri(self, g, lo, hi, shape, dt=None):
        x = self.t.randint(lo, hi, shape, generator=g, device=self.dev, dtype=self.t.int32)
        return x if dt is None else x.to(dt)

    def cst(self, g, W):
        N = W.shape[0]
        c = self.t.zeros((N, 4), dtype=self.t.int32, device=self.dev)
        c[:, 0] = self.ri(g, 16384, 32768, (N,)); c[:, 1] = self.ri(g, 20, 30, (N,)); c[:, 2] = self.ri(g, -50000, 50000, (N,))
        c[:, 3] = W.to(self.t.int32).sum(1)
        return c

    def attention(self):
        """config 2: 8 x 5 heads x 4096 x 4096 x 64 on int16-range activations, the reference's k_fused_attention"""
        torch, P, L = self.t, self.P, self.L
        B, heads, T = ATTN_SHAPE["B"], ATTN_SHAPE["heads"], ATTN_SHAPE["T"]
        C, G, Tp = 64 * heads, B * heads, (T + 127) // 128 * 128
        g = torch.Generator(device=self.dev); g.manual_seed(2)
        X = [self.ri(g, -32768, 32768, (B, T, C)) for _ in range(3)]
        z = lambda *s, dt: torch.zeros(s, dtype=dt, device=self.dev)
        q = [z(G, Tp, 64, dt=torch.int8), z(G, Tp, 64, dt=torch.int8), z(G, Tp, dt=torch.int32)] + [z(G, Tp, dt=torch.int64) for _ in range(3)]
        k = [z(G, Tp, 64, dt=torch.int8), z(G, Tp, 64, dt=torch.int8), z(G, Tp, dt=torch.int32)] + [z(G, Tp, dt=torch.int64) for _ in range(3)]
        v = [z(G, 64, Tp, dt=torch.int8), z(G, 64, Tp, dt=torch.int8), z(G, 64, dt=torch.int32), z(G, 64, dt=torch.int64)]
        self.L.ref_set_sync(1)
        self.ok(L.ref_quant_heads(P(X[0]), B, T, C, heads, Tp, *[P(x) for x in q]))
        self.ok(L.ref_quant_heads(P(X[1]), B, T, C, heads, Tp, *[P(x) for x in k]))
        self.ok(L.ref_quant_v(P(X[2]), B, T, C, heads, Tp, *[P(x) for x in v], P(z(G, 64, dt=torch.int32))))
        self.L.ref_set_sync(0)
        lexp = torch.from_numpy(np.rint(1073741824.0 * np.exp(-np.arange(1025) / 64.0)).astype(np.int64)).to(self.dev)
        gmx, gr = z(G * Tp, dt=torch.int32), z(G * Tp, dt=torch.int64)
        out, rm = z(B, T, C, dt=torch.int32), z(B * T, dt=torch.int32)
        run = lambda: self.ok(L.ref_fused_attention(P(q[0]), P(q[1]), P(q[2]), P(q[3]), P(q[4]), P(k[0]), P(k[1]), P(k[2]), P(k[5]),
                                                    P(v[0]), P(v[1]), P(v[2]), P(v[3]), B, heads, T, Tp, T, Tp, 0, P(lexp), C,
                                                    P(gmx), P(gr), P(out), P(rm)))
        return {"kernel": "reference k_fused_attention (config 2)", "ms": round(self.time(run), 4)}

    def gemm(self):
        """config 1: planar A 4096 x 320 (int16 range), W 320 x 320, the reference's gemm_hl (k_gemm_hl2)"""
        torch, P, L = self.t, self.P, self.L
        M, N, K = 4096, 320, 320
        g = torch.Generator(device=self.dev); g.manual_seed(1)
        q = self.ri(g, -32768, 32768, (M, K))
        hi, lo = (q >> 8).to(torch.int8), ((q & 255) - 128).to(torch.int8)
        W = self.ri(g, -127, 128, (N, K), torch.int8); cst = self.cst(g, W); e = self.ri(g, 0, 12, (M,))
        Y = torch.empty((M, N), dtype=torch.int32, device=self.dev)
        run = lambda: self.ok(L.ref_gemm_hl(P(hi), P(lo), K, M, M, P(W), K, N, N, K, P(cst), P(e), P(Y), N, None, 0, 0, None, None, None, None))
        ms = self.time(run)
        return {"kernel": "reference gemm_hl planar (config 1)", "M": M, "N": N, "K": K, "ms": round(ms, 4), "int8_tops": round(2 * 2 * M * N * K / ms / 1e9, 2)}

    def gn_conv(self, level):
        """config 3: GroupNorm + SiLU of int16-range NHWC [8, H*W, C], then the 3x3 conv C -> C the way the reference's
        engine runs it at these depths (9C > 1536: pixel max, im2col, cuBLASLt, epilogue; src/engine.cu:254-280), and its
        fused-loader gemm_hl (SRC_CONV32) for comparison"""
        torch, P, L = self.t, self.P, self.L
        Hh, C = GnConvCase.LEVELS[level]
        B, T, N, K = 8, Hh * Hh, C, 9 * C
        g = torch.Generator(device=self.dev); g.manual_seed(3)
        X = self.ri(g, -32768, 32768, (B, T, C))
        gam, beta = self.ri(g, 65536 - 16384, 65536 + 16384, (C,)), self.ri(g, -8192, 8192, (C,))
        xs = np.arange(2049, dtype=np.float64) / 64.0 - 16.0
        Lsig = torch.from_numpy(np.rint(65536.0 / (1.0 + np.exp(-xs))).astype(np.int32)).to(self.dev)
        gs = torch.zeros((B * 32, 6), dtype=torch.int64, device=self.dev)
        Y, pm = torch.empty((B, T, C), dtype=torch.int32, device=self.dev), torch.empty((B * T,), dtype=torch.int32, device=self.dev)
        W = self.ri(g, -127, 128, (N, K), torch.int8); cst = self.cst(g, W)
        e = torch.empty((B * T,), dtype=torch.int32, device=self.dev)
        planes = torch.empty((2 * B * T, K), dtype=torch.int8, device=self.dev)
        Cs = torch.empty((2 * B * T, N), dtype=torch.int32, device=self.dev)
        out = torch.empty((B * T, N), dtype=torch.int32, device=self.dev)
        def gn():
            self.ok(L.ref_gn_stats(P(X), B, T, C, 32, 100000, P(gs)))
            self.ok(L.ref_gn_apply_row(P(X), B, T, C, 32, P(gs), P(gam), P(beta), P(Lsig), P(Y), P(pm), None, None, None, 0))
        def conv_lt():
            self.ok(L.ref_pixmax(P(Y), B * T, C, P(pm)))
            self.ok(L.ref_im2col3(P(Y), P(pm), B, Hh, Hh, C, 1, P(planes), self.c.c_void_p(planes.data_ptr() + B * T * K), P(e), K))
            self.ok(L.ref_gemm_lt(P(planes), B * T, B * T, P(W), N, N, K, P(cst), P(e), P(Cs), P(out), N, None))
        def conv_hl():
            self.ok(L.ref_gemm_conv(P(Y), B, Hh, Hh, C, 1, P(pm), P(e), B * T, P(W), K, N, N, K, P(cst), P(out), N, None))
        gn()
        gms, lms, hms = self.time(gn), self.time(conv_lt), self.time(conv_hl)
        ops = 2 * 2 * B * T * N * K
        return {"kernel": "reference GroupNorm+SiLU -> 3x3 conv (config 3)", "B": B, "HW": Hh, "C": C, "gn_ms": round(gms, 4),
                "conv_engine_path_ms": round(lms, 4), "conv_engine_path_int8_tops": round(ops / lms / 1e9, 2),
                "conv_fused_loader_ms": round(hms, 4), "conv_fused_loader_int8_tops": round(ops / hms / 1e9, 2)}

    def norms(self):
        """GroupNorm statistics, GroupNorm + SiLU apply and LayerNorm -> planes at 320 ch 64x64, each timed alone"""
        torch, P, L = self.t, self.P, self.L
        B, T, C = 8, 4096, 320
        g = torch.Generator(device=self.dev); g.manual_seed(3)
        X = self.ri(g, -32768, 32768, (B, T, C))
        gam, beta = self.ri(g, 65536 - 16384, 65536 + 16384, (C,)), self.ri(g, -8192, 8192, (C,))
        xs = np.arange(2049, dtype=np.float64) / 64.0 - 16.0
        Lsig = torch.from_numpy(np.rint(65536.0 / (1.0 + np.exp(-xs))).astype(np.int32)).to(self.dev)
        gs = torch.zeros((B * 32, 6), dtype=torch.int64, device=self.dev)
        Y, pm = torch.empty((B, T, C), dtype=torch.int32, device=self.dev), torch.empty((B * T,), dtype=torch.int32, device=self.dev)
        hi, lo = torch.empty((B * T, C), dtype=torch.int8, device=self.dev), torch.empty((B * T, C), dtype=torch.int8, device=self.dev)
        e = torch.empty((B * T,), dtype=torch.int32, device=self.dev)
        stats = lambda: self.ok(L.ref_gn_stats(P(X), B, T, C, 32, 100000, P(gs)))
        apply = lambda: self.ok(L.ref_gn_apply_row(P(X), B, T, C, 32, P(gs), P(gam), P(beta), P(Lsig), P(Y), P(pm), None, None, None, 0))
        ln = lambda: self.ok(L.ref_lnorm_q(P(X), B * T, C, P(gam), P(beta), 100000, P(hi), P(lo), P(e), C))
        stats()
        ts, ta, tl = self.time(stats), self.time(apply), self.time(ln)
        nb = B * T * C * 4
        return {"kernel": "reference norms (320 ch 64x64)", "gn_stats_ms": round(ts, 4), "gn_stats_gbs": round(2 * nb / ts / 1e6, 1),
                "gn_apply_ms": round(ta, 4), "gn_apply_gbs": round((2 * nb + B * T * 4) / ta / 1e6, 1),
                "lnorm_q_ms": round(tl, 4), "lnorm_q_gbs": round((nb + nb // 2) / tl / 1e6, 1)}

    def linear(self, kind, K):
        """the UNet's 64x64-level linears: int32 input quantised on load (K 320 / 1280, N 320, + residual + row max), the GEGLU
        GEMM (K 320, N 2560), the merged q|k|v GEMM with head quantisation (K 320, N 960); the reference's gemm_hl forms"""
        torch, P, L = self.t, self.P, self.L
        M = 32768
        N = {"geglu": 2560, "qkv": 960}.get(kind, 320)
        g = torch.Generator(device=self.dev); g.manual_seed(4)
        W = self.ri(g, -127, 128, (N, K), torch.int8); cst = self.cst(g, W)
        if kind == "linear":
            X = self.ri(g, -(1 << 20), 1 << 20, (M, K)); rm = X.abs().amax(1).to(torch.int32)
            R = self.ri(g, -(1 << 20), 1 << 20, (M, N)); Y = torch.empty((M, N), dtype=torch.int32, device=self.dev)
            rmo = torch.zeros((M,), dtype=torch.int32, device=self.dev)
            run = lambda: self.ok(L.ref_gemm_x32(P(X), K, P(rm), K, M, M, P(W), K, N, N, K, P(cst), P(Y), N, P(R), 0, None, P(rmo)))
        else:
            q = self.ri(g, -32768, 32768, (M, K)); hi, lo = (q >> 8).to(torch.int8), ((q & 255) - 128).to(torch.int8); e = self.ri(g, 0, 6, (M,))
            if kind == "geglu":
                from math import erf, sqrt
                xs = np.arange(2049, dtype=np.float64) / 64.0 - 16.0
                Lphi = torch.from_numpy(np.rint([65536.0 * 0.5 * (1 + erf(x / sqrt(2))) for x in xs]).astype(np.int32)).to(self.dev)
                Y = torch.empty((M, N // 2), dtype=torch.int32, device=self.dev); rmo = torch.zeros((M,), dtype=torch.int32, device=self.dev)
                run = lambda: self.ok(L.ref_gemm_hl(P(hi), P(lo), K, M, M, P(W), K, N, N, K, P(cst), P(e), P(Y), N // 2, None, 2, 0, None, None, P(Lphi), P(rmo)))
            else:
                heads, T, C = 5, 4096, 320
                G, Tp = (M // T) * heads, T
                z = lambda *s, dt: torch.zeros(s, dtype=dt, device=self.dev)
                qb = [z(G, Tp, 64, dt=torch.int8), z(G, Tp, 64, dt=torch.int8), z(G, Tp, dt=torch.int32)] + [z(G, Tp, dt=torch.int64) for _ in range(3)]
                kb = [z(G, Tp, 64, dt=torch.int8), z(G, Tp, 64, dt=torch.int8), z(G, Tp, dt=torch.int32)] + [z(G, Tp, dt=torch.int64) for _ in range(3)]
                V = z(M, C, dt=torch.int32)
                run = lambda: self.ok(L.ref_gemm_qkv(P(hi), P(lo), K, P(e), M, M, P(W), K, N, N, K, P(cst), heads, T, Tp, Tp, C,
                                                     *[P(x) for x in qb], *[P(x) for x in kb], P(V)))
        ms = self.time(run)
        return {"kernel": f"reference gemm_hl {kind} (64x64 level)", "M": M, "N": N, "K": K, "ms": round(ms, 4), "int8_tops": round(2 * 2 * M * N * K / ms / 1e9, 2)}


# ------------------------------------------------------------------ CPU baseline (the oracle, bounded sample)
def cpu_baseline(path):
    from oracle import pyoracle as O
    from vela_b200.dist import golden_seeds
    cores = os.cpu_count() or 1
    O.lib().or_set_threads(cores)
    m = O.Model(path)
    m.set_prompt(PROMPT)
    t0 = time.perf_counter()
    m.step(golden_seeds(1))
    dt = time.perf_counter() - t0
    m.close()
    return {"value": 1.0 / dt, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"one UNet step at batch 1 (1 of the 16 inferences of a GPU step) on the oracle's C restatement, "
                      f"OpenMP x {cores} threads: {dt:.2f} s"}


# ------------------------------------------------------------------ our arm
def run_vela(a, R):
    import torch
    import vela_b200 as V
    from vela_b200.dist import seed_block, golden_seeds
    dev = torch.device("cuda", R.local)
    path = model_file(R, "product")
    model = V.Model(path, R.local)
    lanes = [V.Engine(model, batch=a.batch, graph=True) for _ in range(a.lanes)]
    for e in lanes:
        e.set_prompt(PROMPT)

    # parity of the bench's own engine: golden seeds -> the reference engine's x0 (tests/golden/engine.npz)
    gs = golden_seeds(a.batch)
    x0 = lanes[0].run(gs)
    gold = np.load(os.path.join(ROOT, "tests", "golden", "engine.npz"))
    ref_ok = bool(np.array_equal(x0[: len(gold["x0"])], gold["x0"]))
    same = R.agree(hashlib.sha256(x0.tobytes()).digest())

    # device-resident inputs: seeds of every (rank, lane, step) already in HBM
    n_steps = a.warmup + a.steps
    seeds = torch.from_numpy(np.stack([np.stack([seed_block(R.rank, l, s, a.batch) for s in range(n_steps)]) for l in range(a.lanes)])).to(dev)
    out = torch.empty((a.lanes, a.batch, 32768), dtype=torch.uint8, device=dev)
    streams = [torch.cuda.ExternalStream(e.stream, device=dev) for e in lanes]
    main = torch.cuda.current_stream(dev)

    def launch(step):
        for l, e in enumerate(lanes):
            e.launch_device(seeds[l, step].data_ptr(), out[l].data_ptr())

    for s in range(a.warmup):
        launch(s)
    torch.cuda.synchronize(dev)
    kernels_per_step = sum(e.graph_kernels for e in lanes)
    R.barrier(); torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ends = [torch.cuda.Event() for _ in lanes]
    with Clocks(R.local) as clk:
        e0.record(main)
        for st in streams:
            st.wait_event(e0)
        for s in range(a.steps):
            launch(a.warmup + s)
        for st, ev in zip(streams, ends):
            ev.record(st)
            main.wait_event(ev)
        e1.record(main)
        torch.cuda.synchronize(dev)
    R.barrier()
    ms = R.max(e0.elapsed_time(e1))
    assert V.lib().vela_device_error(1) == 0, "a kernel reported a device error"
    # the device-resident path computes what the host path computes
    dev_ok = bool(np.array_equal(out[0].cpu().numpy(), lanes[0].run(seeds[0, a.warmup + a.steps - 1].cpu().numpy())))
    per_step = a.lanes * a.batch
    value = R.world * per_step * a.steps / (ms / 1000.0)

    e2e = None
    if not a.no_e2e:
        host = [[seed_block(R.rank, l, 10_000 + s, a.batch) for s in range(a.steps + a.warmup)] for l in range(a.lanes)]
        outs = [np.empty((a.batch, 32768), np.uint8) for _ in lanes]

        def lane_loop(l, first, count):
            e = lanes[l]
            e.submit(host[l][first])
            for i in range(count):
                if i + 1 < count:
                    e.submit(host[l][first + i + 1])
                e.collect(outs[l])

        def run_threads(first, count):
            th = [threading.Thread(target=lane_loop, args=(l, first, count)) for l in range(a.lanes)]
            for t in th:
                t.start()
            for t in th:
                t.join()

        run_threads(0, a.warmup)
        R.barrier(); torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        run_threads(a.warmup, a.steps)
        torch.cuda.synchronize(dev)
        sec = R.max(time.perf_counter() - t0)
        R.barrier()
        e2e = {"value": R.world * per_step * a.steps / sec, "unit": UNIT,
               "h2d_bytes_per_step": per_step * 32, "d2h_bytes_per_step": per_step * 32768,
               "bytes_scope": "per GPU per step (seeds in, x0 out)", "timing": "host wall clock between barriers, max over ranks"}

    roof = None
    if not a.no_roofline:
        case = AttentionCase(dev)
        ams = case.time_ms()
        hbm, bf16, src = peaks()
        peak = 2.0 * bf16
        achieved = ATTN_OPS / (ams / 1000.0) / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                "traffic": profile_traffic(), "kernel": "attn_kernel (vela_fused_attention), self-attention 8 x 5 heads x 4096 x 64",
                "ms_per_launch": round(ams, 3), "ops_per_launch": ATTN_OPS,
                "peak_note": f"int8 dense ops/s = 2 x the {src} bf16 burst GEMM rate; ops are single-pass algorithmic (the exact "
                             f"3-pass algorithm executes the QK products twice more)"}
        del case

    cpu = None
    if R.world == 1 and R.rank == 0 and not a.no_cpu_baseline:
        cpu = cpu_baseline(path)

    for e in lanes:
        e.close()
    model.close()
    if R.rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": R.world, "steps": a.steps, "warmup": a.warmup,
                "ms_per_step": round(ms / a.steps, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "int8 MMA / int32-int64", "data": "synthetic: seeded random-init int8 POISD model, ChaCha20 noise from per-(gpu, lane, step) seeds",
                "config": {"workload": "one SD-turbo UNet denoising step (noise -> UNet -> x0) per inference, batch 8 x 2 lanes per GPU, "
                                       "one CUDA graph per lane step", "batch": a.batch, "lanes": a.lanes, "inferences_per_step_per_gpu": per_step,
                           "prompt_tokens": PROMPT, "l2": "inputs larger than L2: 1.4 GB of weights and ~2 GB of activations stream per step"},
                "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": kernels_per_step * a.steps * R.world, "kernels_per_step_per_gpu": kernels_per_step,
                "clocks": clk.summary(), "x0_matches_reference_engine": ref_ok, "x0_same_on_all_ranks": same, "device_path_matches_host_path": dev_ok}
        print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ reference arm
def run_reference(a, R):
    import ctypes
    import torch
    so = os.path.join(ROOT, "oracle", "_ref", "libvela_ref.so")
    if not os.path.exists(so):
        if R.rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libvela_ref.so (the reference built from its sources) is missing; "
                                                                  "build it with `make -C oracle ref` where the reference checkout is present"}), flush=True)
        return
    path = model_file(R, "oracle")
    L = ctypes.CDLL(so)
    L.ref_open.restype = ctypes.c_void_p
    L.ref_open.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    L.ref_set_prompt.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    L.ref_bench.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_longlong)]
    L.ref_close.argtypes = [ctypes.c_void_p]
    L.ref_last_error.restype = ctypes.c_char_p
    h = L.ref_open(path.encode(), R.local, a.batch, a.lanes, 1)
    if not h:
        raise RuntimeError("reference engine: " + L.ref_last_error().decode())
    toks = (ctypes.c_int * len(PROMPT))(*PROMPT)
    if L.ref_set_prompt(h, toks, len(PROMPT)) != 0:
        raise RuntimeError("reference set_prompt: " + L.ref_last_error().decode())
    sec, inf = ctypes.c_double(), ctypes.c_longlong()
    # warm-up inside ref_bench (two batches per lane per warm-up step); then K steps per lane, one host thread per lane
    R.barrier(); torch.cuda.synchronize()
    with Clocks(R.local) as clk:
        if L.ref_bench(h, a.warmup, a.steps, ctypes.byref(sec), ctypes.byref(inf)) != 0:
            raise RuntimeError("reference bench: " + L.ref_last_error().decode())
    R.barrier()
    s = R.max(sec.value)
    L.ref_close(h)
    # the CPU figure beside it: the reference has no CPU implementation of the path, so this is the oracle's C
    # restatement of its integer spec (kind "port"), the same bounded sample as our arm's
    cpu = cpu_baseline(path) if R.world == 1 and R.rank == 0 and not a.no_cpu_baseline else None
    if R.rank == 0:
        per_step = a.lanes * a.batch
        value = R.world * per_step * a.steps / s
        line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": R.world, "steps": a.steps, "warmup": a.warmup,
                "ms_per_step": round(s * 1000.0 / a.steps, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "int8 MMA / int32-int64", "data": "synthetic: the same seeded random-init int8 POISD model and prompt",
                "config": {"workload": "one SD-turbo UNet denoising step (noise -> UNet -> x0) per inference, batch 8 x 2 lanes per GPU, "
                                       "one CUDA graph per lane step", "batch": a.batch, "lanes": a.lanes, "inferences_per_step_per_gpu": per_step,
                           "prompt_tokens": PROMPT, "l2": "inputs larger than L2: 1.4 GB of weights and ~2 GB of activations stream per step"},
                "impl": "reference",
                "reference_kind": "gpu",
                "reference_run": f"the reference engine compiled from its own sources for sm_100 (oracle/_ref/libvela_ref.so, cuBLASLt + "
                                 f"mma.sync kernels, default EngineConfig): Engine::submit/collect from {a.lanes} host threads per GPU "
                                 f"(src/main.cpp:111-162), {a.steps} steps per lane after {a.warmup} warm-up steps, on the same model bytes "
                                 f"(written by oracle/synth_model.c), prompt, batch and lanes as our arm",
                "cpu_baseline": cpu,
                "native_libs": loaded_native_libs(),
                "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": per_step * 32, "d2h_bytes_per_step": per_step * 32768},
                "clocks": clk.summary()}
        print(json.dumps(line), flush=True)


def run_kernel(a, R):
    import torch
    dev = torch.device("cuda", R.local)
    if a.impl == "reference":
        K = RefKernels(dev)
        if a.kernel == "attention":
            rep = K.attention()
        elif a.kernel == "gemm":
            rep = K.gemm()
        elif a.kernel == "norms":
            rep = K.norms()
        elif a.kernel in ("linear", "geglu", "qkv"):
            rep = K.linear(a.kernel, a.linear_k if a.kernel == "linear" else 320)
        else:
            rep = K.gn_conv(a.conv_level)
        torch.cuda.synchronize()
        rep["impl"] = "reference"
        rep["native_libs"] = loaded_native_libs()
        if R.rank == 0:
            print(json.dumps(rep), flush=True)
        return
    if a.kernel == "attention":
        case = AttentionCase(dev)
        for _ in range(3):
            case.launch()
        rep = {"kernel": "attention (config 2)", "ms": round(case.time_ms(), 4)}
    elif a.kernel == "gemm":
        case = GemmCase(dev)
        rep = case.report()
    elif a.kernel == "norms":
        case = GnConvCase(dev, 0)
        rep = case.report_norms()
    elif a.kernel in ("linear", "geglu", "qkv"):
        case = LinearCase(dev, a.kernel, a.linear_k if a.kernel == "linear" else 320)
        rep = case.report()
    else:
        case = GnConvCase(dev, a.conv_level)
        rep = case.report()
    torch.cuda.synchronize()
    assert case.L.vela_device_error(1) == 0, "a kernel reported a device error"
    if R.rank == 0:
        print(json.dumps(rep), flush=True)


def main():
    a = parse()
    R = Ranks()
    R.init()
    try:
        if a.kernel:
            run_kernel(a, R)
        elif a.impl == "reference":
            run_reference(a, R)
        else:
            run_vela(a, R)
    finally:
        R.close()


if __name__ == "__main__":
    main()
