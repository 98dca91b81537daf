"""Benchmark of the WKV-7 / quantised-GEMV hot paths on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Prints ONE JSON line (rank 0).  Under torchrun (N > 1) every rank runs its own
replica of the workload (the paths shard with no exchange), timing is the max
over ranks and `value` counts the units of all ranks.

Workloads (synthetic, seeded 0x5EED2026):
  decode   config 4 (default) -- random-init x070 1.5B (L=24, C=2048, H=32,
           vocab 65536, FFN 8192) over a 4-bit group-64 base, fp16
           activations; `--rows` rows per GPU (default 64) each prefilled
           with 128 uniform-random tokens, then greedy decode steps through
           the captured CUDA graph; tok/s = rows per step.  Weights (0.86 GB)
           and state (25 MB per row) exceed L2, so no flush is needed.
  wkv7     config 1 -- WKV-7 operator forward, B=1 T=1024 H=12 N=64 fp32,
           tok/s = B*T per step.  Inputs (22 MB) are smaller than L2, so L2 is
           flushed (a 256 MB write) before every timed step, outside the timed
           interval.
  wkv7train  config 1 as the operator row of the survey measures it:
           forward + backward of the training path (chunked train forward
           with 16-token checkpoints, chunked DPLR backward), dy ~ N(0,1);
           tok/s = B*T per step; L2 flushed before every timed step.
  gemv     config 2 -- 4-bit g64 GEMV over the four 1.5B projection shapes,
           rows 1, fp16 activations; GB/s of the packed weight stream.
  statetune  config 5 on the WKV path -- the per-layer initial states of
           x070 2.9B (L=32, H=40) trained by WKVStateTuner on one 4096-token
           sequence per GPU (data-parallel under torchrun: NCCL allreduce of
           the state gradients), clip + AdamW on the device; tok/s.
`--impl reference` times the CPU oracle (the reference's Metal/MLX path
cannot run here) on the same workload and metric, on all host cores.
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

# The CPU legs run the oracle's OpenMP loops on every host core.  The few small
# numpy matmuls they also make get one BLAS thread, set before numpy loads
# OpenBLAS: a BLAS pool of one thread per core spinning beside the OpenMP pool
# slowed the CPU decode baseline ~40x when nothing capped it (under torchrun
# OMP_NUM_THREADS=1 capped it, so N=1 and N>1 disagreed).
BLAS_THREADS = 1
os.environ.setdefault("OPENBLAS_NUM_THREADS", str(BLAS_THREADS))
os.environ.setdefault("MKL_NUM_THREADS", str(BLAS_THREADS))

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
SEED = 0x5EED2026


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


def measured_traffic(wl):
    """DRAM bytes (read + write) per launch of the dominant kernel, from the
    ncu capture summarised in profiles/traffic.json for this workload and row
    count; None when no capture covers it."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p) or getattr(wl, "rq_kind", None) or getattr(wl, "persistent", False):
        return None  # the captures cover the 4-bit per-op kernels only
    with open(p) as f:
        d = json.load(f)
    e = d.get(wl.name, {}).get(str(getattr(wl, "rows", "")))
    return None if e is None else e["dram_bytes_per_launch"]


# ---------------------------------------------------------------- clock sampling

class ClockSampler:
    """nvidia-smi SM clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() in ("active", "1"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# -------------------------------------------------------------------- workloads

def config1_inputs(rng, B=1, T=1024, H=12, N=64):
    def n():
        return rng.standard_normal((B, T, H, N)).astype(np.float32)
    r, k, v = n(), n(), n()
    u = -np.logaddexp(0, -n()) - 0.5
    w = np.exp(-np.exp(u)).astype(np.float32)
    kk = n()
    kk /= np.sqrt((kk * kk).sum(-1, keepdims=True))
    a = (-kk).astype(np.float32)
    b = (kk / (1 + np.exp(-n()))).astype(np.float32)
    return [r, w, k, v, a, b]


class WKV7Prefill:
    name = "wkv7"
    metric = ("WKV-7 prefill tok/s (config 1 operator forward, B=1 T=1024 H=12 N=64 fp32, "
              "chunked DPLR form)")
    unit = "tok/s"
    B, T, H, N = 1, 1024, 12, 64

    def setup(self, torch, dev):
        from swiftrwkv_b200 import _lib
        self.torch, self._lib = torch, _lib
        rng = np.random.default_rng(SEED)
        self.host = config1_inputs(rng, self.B, self.T, self.H, self.N)
        self.x = [torch.from_numpy(a).to(dev) for a in self.host]
        self.y = torch.empty_like(self.x[0])
        self.h = torch.empty((self.B, self.H, self.N, self.N), device=dev)
        self.pin = [torch.from_numpy(a).pin_memory() for a in self.host]
        self.pin_y = torch.empty(self.y.shape, dtype=torch.float32).pin_memory()
        self.units_per_step = self.B * self.T
        # chunked form: prep (chunk transitions), scan, out
        self.launches_per_step = 3
        ws_bytes = int(_lib.lib().rwkv_wkv7_forward_chunked_workspace_size(self.B, self.T, self.H, self.N))
        self.ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        self.ws_bytes = ws_bytes
        # algorithmic bytes: 6 inputs + y (fp32) + h_out (h_in = 0 is not read)
        BTHN = self.B * self.T * self.H * self.N
        self.alg_bytes = 4 * (7 * BTHN + self.B * self.H * self.N * self.N)
        self.kernel = "wkv7_chunk_{prep,scan,out} (per launch: the three-kernel step / 3)"
        self.h2d = sum(a.nbytes for a in self.host)
        self.d2h = self.y.numel() * 4

    def step(self):
        _lib, P = self._lib, self._lib.P
        st = P(self.torch.cuda.current_stream().cuda_stream)
        _lib.call("rwkv_wkv7_forward_chunked", 0, *(P(t.data_ptr()) for t in self.x), None,
                  P(self.y.data_ptr()), P(self.h.data_ptr()), None, self.B, self.T, self.H, self.N,
                  P(self.ws.data_ptr()), self.ws_bytes, st)

    def step_e2e(self):
        for d, p in zip(self.x, self.pin):
            d.copy_(p, non_blocking=True)
        self.step()
        self.pin_y.copy_(self.y, non_blocking=True)

    def cpu(self, seconds):
        from oracle import oracle as O
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < seconds or n == 0:
            O.wkv7_forward(*self.host)
            n += 1
        dt = time.perf_counter() - t0
        return n * self.B * self.T / dt, f"{n} full config-1 forwards ({n * self.B * self.T} tokens)"


class WKV7Train:
    """Config 1 as SURVEY's operator row measures it: forward + backward of the
    WKV-7 training path (chunked train forward with checkpoints, chunked DPLR
    backward), B=1 T=1024 H=12, dy ~ N(0,1)."""
    name = "wkv7train"
    metric = ("WKV-7 forward + backward tok/s (config 1 operator, B=1 T=1024 H=12 N=64 fp32, "
              "chunked DPLR train forward + backward)")
    unit = "tok/s"
    B, T, H, N = 1, 1024, 12, 64

    def setup(self, torch, dev):
        from swiftrwkv_b200 import _lib
        self.torch, self._lib = torch, _lib
        rng = np.random.default_rng(SEED)
        self.host = config1_inputs(rng, self.B, self.T, self.H, self.N)
        self.host.append(rng.standard_normal(self.host[0].shape).astype(np.float32))   # dy
        self.x = [torch.from_numpy(a).to(dev) for a in self.host]
        shp = (self.B, self.T, self.H, self.N)
        self.y = torch.empty(shp, device=dev)
        self.ck = torch.empty((self.B, self.H, self.T // 16, self.N, self.N), device=dev)
        self.g = [torch.empty(shp, device=dev) for _ in range(6)]
        self.dh = torch.empty((self.B, self.H, self.N, self.N), device=dev)
        L = _lib.lib()
        self.ws_bytes = max(int(L.rwkv_wkv7_forward_chunked_workspace_size(self.B, self.T, self.H, self.N)),
                            int(L.rwkv_wkv7_backward_chunked_workspace_size(self.B, self.T, self.H, self.N)))
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=dev)
        self.pin = [torch.from_numpy(a).pin_memory() for a in self.host]
        self.pin_g = [torch.empty(shp, dtype=torch.float32).pin_memory() for _ in range(6)]
        self.units_per_step = self.B * self.T
        # forward: prep, scan, out; backward: prep, reverse scan, out
        self.launches_per_step = 6
        BTHN = self.B * self.T * self.H * self.N
        BHN2 = self.B * self.H * self.N * self.N
        # canonical bytes: forward 4(7 BTHN + 2 BHN^2) + backward 4(14 BTHN + 3 BHN^2)
        self.alg_bytes = 4 * (21 * BTHN + 5 * BHN2)
        self.kernel = ("wkv7_chunk_{prep,scan,out} + wkv7_chunk_bwd_{prep,out} + reverse scan "
                       "(per launch: the six-kernel step / 6)")
        self.h2d = sum(a.nbytes for a in self.host)
        self.d2h = 6 * BTHN * 4

    def step(self):
        _lib, P = self._lib, self._lib.P
        st = P(self.torch.cuda.current_stream().cuda_stream)
        r, w, k, v, a, b, dy = (P(t.data_ptr()) for t in self.x)
        ws = P(self.ws.data_ptr())
        _lib.call("rwkv_wkv7_train_forward_chunked", 0, r, w, k, v, a, b, None, P(self.y.data_ptr()), None,
                  None, P(self.ck.data_ptr()), self.B, self.T, self.H, self.N, ws, self.ws_bytes, st)
        _lib.call("rwkv_wkv7_backward_chunked", 0, r, w, k, v, a, b, None, P(self.ck.data_ptr()), dy, None,
                  *(P(t.data_ptr()) for t in self.g), P(self.dh.data_ptr()), self.B, self.T, self.H, self.N,
                  ws, self.ws_bytes, st)

    def step_e2e(self):
        for d, p in zip(self.x, self.pin):
            d.copy_(p, non_blocking=True)
        self.step()
        for h, d in zip(self.pin_g, self.g):
            h.copy_(d, non_blocking=True)

    def cpu(self, seconds):
        from oracle import oracle as O
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < seconds or n == 0:
            O.wkv7_train(*self.host[:6], None, self.host[6])
            n += 1
        dt = time.perf_counter() - t0
        return n * self.B * self.T / dt, f"{n} full config-1 forward + backward passes ({n * self.B * self.T} tokens)"


class GemvSuite:
    name = "gemv"
    unit = "GB/s"
    MATS = [(2048, 2048), (8192, 2048), (2048, 8192), (65536, 2048)]

    def __init__(self, rows=1):
        self.rows = rows
        self.metric = (f"4-bit g64 GEMV GB/s (config 2, 1.5B projection shapes, rows {rows}, "
                       "fp16 x)")

    def setup(self, torch, dev):
        from swiftrwkv_b200 import _lib
        self.torch, self._lib = torch, _lib
        g = torch.Generator(device="cpu").manual_seed(SEED)
        self.mats = []
        from swiftrwkv_b200 import quant as Q
        for OUT, IN in self.MATS:
            W = (torch.randn((OUT, IN), generator=g) * 0.02).half().to(dev)
            wq, sc, bi = Q.quantized(W)
            x = torch.randn((self.rows, IN), generator=g).half().to(dev)
            y = torch.empty((self.rows, OUT), device=dev, dtype=torch.float32)
            self.mats.append((OUT, IN, wq, sc, bi, x, y))
            del W
        R = self.rows
        mat_bytes = lambda OUT, IN: OUT * IN * 0.5 + OUT * IN // 64 * 4 + R * IN * 2 + R * OUT * 4
        self.alg_bytes = sum(mat_bytes(OUT, IN) for OUT, IN in self.MATS)
        self.units_per_step = self.alg_bytes / 1e9
        self.launches_per_step = len(self.MATS)
        # the dominant launch: the 65536 x 2048 head matrix
        self.dom_bytes = mat_bytes(*self.MATS[-1])
        self.kernel = ("q4_gemv_stream_kernel (streaming CUDA-core GEMV, x staged once per CTA), 65536x2048"
                       if R <= 2 else
                       "gemm_w4_kernel (mma.sync GEMV mode, exact per-group scaling), 65536x2048"
                       if R <= 8 else "gemm_tc_kernel (tcgen05, TMA + TMEM), 65536x2048")
        self.h2d = sum(R * IN * 2 for _, IN in self.MATS)
        self.d2h = sum(R * OUT * 4 for OUT, _ in self.MATS)
        self.pin_x = [torch.empty((R, IN), dtype=torch.float16).pin_memory() for _, IN in self.MATS]
        self.pin_y = [torch.empty((R, OUT), dtype=torch.float32).pin_memory() for OUT, _ in self.MATS]

    def _gemm(self, OUT, IN, wq, sc, bi, x, y):
        _lib, P = self._lib, self._lib.P
        st = P(self.torch.cuda.current_stream().cuda_stream)
        _lib.call("rwkv_q_gemm", 2, P(x.data_ptr()), P(wq.data_ptr()), P(sc.data_ptr()),
                  P(bi.data_ptr()), 2, 0, P(y.data_ptr()), self.rows, OUT, IN, 64, 4, st)

    def step(self):
        for m in self.mats:
            self._gemm(*m)

    def dominant(self):
        self._gemm(*self.mats[-1])

    def step_e2e(self):
        for (OUT, IN, wq, sc, bi, x, y), px, py in zip(self.mats, self.pin_x, self.pin_y):
            x.copy_(px, non_blocking=True)
        self.step()
        for (OUT, IN, wq, sc, bi, x, y), py in zip(self.mats, self.pin_y):
            py.copy_(y, non_blocking=True)

    def cpu(self, seconds):
        from oracle import oracle as O
        rng = np.random.default_rng(SEED)
        OUT, IN = 2048, 2048
        W = (rng.standard_normal((OUT, IN)) * 0.02).astype(np.float16).astype(np.float32)
        wq, sc, bi = O.affine_quantize(W)
        x = rng.standard_normal((1, IN)).astype(np.float16).astype(np.float32)
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < seconds or n == 0:
            O.affine_gemv(x, wq, sc, bi)
            n += 1
        dt = time.perf_counter() - t0
        by = OUT * IN * 0.5 + OUT * IN // 64 * 4
        return n * by / dt / 1e9, f"{n} GEMVs of 2048x2048 4-bit g64, 1 row"


class Decode15B:
    name = "decode"
    unit = "tok/s"
    L, C, V, PROMPT = 24, 2048, 65536, 128

    # --base: the projection / head matrices' container.  q4: MLX affine 4-bit
    # group 64 (config 4's QLoRA base); sb6 / sym6 / sym8: .rwkvq matrices kept
    # native (rwkv_x070_set_param_rwkvq), the formats of the reference's
    # published decode timings (docs/Inference.md:550-557: "compression" = sb6,
    # "reduction" = sym); synthetic codes and scales.
    BASES = {"q4": ("MLX affine 4-bit g64", None, 0),
             "sb6": (".rwkvq sb6 5-bit (4 + 1 bit-plane, group 32; compression)", "sb6", 1),
             "sym6": (".rwkvq sym 6-bit (reduction)", "sym", 6),
             "sym8": (".rwkvq sym 8-bit (reduction)", "sym", 8)}

    def __init__(self, rows=64, prompt=128, decode_path="launches", base="q4"):
        self.rows = rows
        self.PROMPT = prompt
        self.decode_path = decode_path
        self.base = base
        self.base_label, self.rq_kind, self.rq_bits = self.BASES[base]
        what = "4-bit" if base == "q4" else self.base_label
        self.metric = (f"x070 1.5B {what} decode tok/s (generateBatch greedy, {rows} rows/GPU, "
                       "fp16 activations)")

    def _matrices(self):
        C, F, V = self.C, 4 * self.C, self.V
        for l in range(self.L):
            for n in ("tmix.r_proj", "tmix.k_proj", "tmix.v_proj", "tmix.o_proj"):
                yield f"blocks.{l}.{n}.weight", C, C
            yield f"blocks.{l}.cmix.key.weight", F, C
            yield f"blocks.{l}.cmix.value.weight", C, F
        yield "head.weight", V, C

    def _set_rwkvq(self):
        """Every projection and the head as native .rwkvq matrices (synthetic
        codes, small positive scales); returns the bytes they replace and add."""
        import ctypes
        from swiftrwkv_b200 import _lib
        rng = np.random.default_rng(SEED)
        kind, bits = self.rq_kind, self.rq_bits
        old = new = 0
        for key, OUT, IN in self._matrices():
            if kind == "sb6":
                NB = IN // 32
                b1 = rng.integers(0, 256, OUT * NB * (16 + 4 * bits), dtype=np.uint8)
                b2 = rng.integers(0, 64, OUT * NB * 2, dtype=np.uint8)
                b3 = (rng.random(OUT * (IN // 256) * 2) * 1e-3).astype(np.float16)
                fmt = 1
            else:
                b1 = rng.integers(0, 256, OUT * IN if bits == 8 else OUT * IN // 32 * 24, dtype=np.uint8)
                b2 = rng.integers(0, 128, OUT * IN // 16, dtype=np.uint8)
                b3 = (rng.random(OUT * (IN // 256)) * 1e-4).astype(np.float16)
                fmt = 2
            args = []
            for b in (b1, b2, b3):
                args += [b.ctypes.data_as(ctypes.c_void_p), b.nbytes]
            _lib.call("rwkv_x070_set_param_rwkvq", self.m.h, key.encode(), fmt, bits, *args)
            old += OUT * IN * (0.5 + 4 / 64)
            new += RwkvqGemvSuite.wbytes(kind, bits, OUT, IN)
        return old, new

    def setup(self, torch, dev):
        from swiftrwkv_b200.x070 import X070Backbone, X070Config
        self.torch = torch
        cfg = X070Config(self.L, self.C, self.V)
        self.m = X070Backbone(cfg, max_rows=self.rows, act="f16").init_random(seed=SEED)
        self.rq_bytes = (0, 0)
        if self.rq_kind:
            self.rq_bytes = self._set_rwkvq()
        self.m.set_decode_path(1 if self.decode_path == "persistent" else 0)
        self.stream = torch.cuda.Stream(device=dev)
        torch.cuda.set_stream(self.stream)
        rng = np.random.default_rng(SEED)
        prompts = rng.integers(0, self.V, (self.rows, self.PROMPT), dtype=np.int32)
        self.m.reset(self.rows)
        for t in range(self.PROMPT):
            self.m.step_greedy(self.rows, torch.from_numpy(prompts[:, t].copy()).to(dev))
        torch.cuda.synchronize()
        H = self.C // 64
        self.state_bytes = self.rows * self.L * H * 64 * 64 * 4 * 2   # read + write
        shift_bytes = self.rows * self.L * self.C * 4 * 2 * 2
        self.alg_bytes = self.m.weight_bytes - self.rq_bytes[0] + self.rq_bytes[1] + self.state_bytes + shift_bytes
        self.units_per_step = self.rows
        self.launches_per_step = self.m.launches_per_step
        # e2e: the previous step's tokens go host -> device, this step's
        # argmax comes back to the host, which waits for it (as generate does)
        self.pin_ids = torch.from_numpy(prompts[:, -1].copy()).pin_memory()
        self.pin_out = torch.zeros(self.rows, dtype=torch.int32).pin_memory()
        self.dev_ids = torch.zeros(self.rows, dtype=torch.int32, device=dev)
        self.dev_next = torch.zeros(self.rows, dtype=torch.int32, device=dev)
        self.h2d = self.rows * 4
        self.d2h = self.rows * 4
        self.persistent = bool(self.m.decode_path(self.rows))
        if self.persistent:
            # one cooperative launch per step: the kernel is the whole step
            self.launches_per_step = 1
            self.dom_bytes = self.alg_bytes
            bn = 16 if self.rows <= 16 else 32 if self.rows <= 32 else 64
            self.kernel = (f"x070_persist_kernel<{bn}> (the whole decode step in one cooperative launch: "
                           "24 layers' 4-bit and low-rank projections on tcgen05, WKV step + tail, glue, head, "
                           "argmax; algorithmic bytes = the step's weights + state read/write + shift rows)")
        else:
            self._family()

    def _family(self):
        """The dominant kernel family: the 4-bit projection GEMMs of the step
        (r/k/v, o, key, value in every layer, and the head)."""
        R, C, F, V, L = self.rows, self.C, 4 * self.C, self.V, self.L
        q = lambda OUT, IN: OUT * IN * (0.5 + 4 / 64)
        if self.rq_kind:
            q = lambda OUT, IN: RwkvqGemvSuite.wbytes(self.rq_kind, self.rq_bits, OUT, IN)
        self.family = {
            "gemm_rkv": 3 * (q(C, C) + R * C * 2 + R * C * 4),
            "gemm_o": q(C, C) + R * C * 2 + R * C * 8,          # y += : read + write
            "gemm_key": q(F, C) + R * C * 2 + R * F * 2,        # relu^2 out fp16
            "gemm_value": q(C, F) + R * F * 2 + R * C * 8,
            "gemm_head": q(V, C) + R * C * 2 + R * V * 4,
        }
        self.family_launches = 4 * L + 1
        self.dom_bytes = (L * sum(v for k, v in self.family.items() if k != "gemm_head")
                          + self.family["gemm_head"]) / self.family_launches
        kern = ("gemm_tc_kernel<TC_Q4> (tcgen05 4-bit GEMM, TMA + TMEM)" if R > 8 else
                "q4_gemv_stream_kernel (streaming CUDA-core 4-bit GEMV)" if R <= 2 else
                "gemm_w4_kernel (mma.sync 4-bit GEMV mode)")
        if self.rq_kind:
            kern = f"{self.rq_kind}_gemv_tile_kernel (.rwkvq {self.base} GEMV, launches of up to 4 rows)"
        self.kernel = (f"{kern}: r/k/v, o, key, value x {L} layers + head = {self.family_launches} "
                       "launches per step; per-launch time from the runtime's step profiler "
                       "(rwkv_x070_profile_step: an event after every launch of a captured step)")

    def step(self):
        self.m.step_greedy(self.rows, None, use_graph=True)

    def step_e2e(self):
        self.dev_ids.copy_(self.pin_ids, non_blocking=True)
        self.m.step_greedy(self.rows, self.dev_ids, use_graph=True, next_ids=self.dev_next)
        self.pin_out.copy_(self.dev_next, non_blocking=True)
        self.torch.cuda.current_stream().synchronize()
        self.pin_ids.copy_(self.pin_out)

    def dominant_ms(self, reps):
        """Average device time per launch of the dominant kernel family inside
        the step: the persistent step kernel, or the 4-bit GEMM launches."""
        if self.persistent:
            # the step profiler times the kernel's phases (grid barrier to grid barrier)
            ts, ph = [], {}
            for _ in range(reps):
                agg, seq = self.m.profile_step(self.rows)
                if not seq:
                    raise RuntimeError("step profiler returned no phases")
                ts.append(sum(t for _, t in seq))
                for name, (c, t) in agg.items():
                    pc, pt = ph.get(name, (0, 0.0))
                    ph[name] = (pc + c, pt + t)
            # per phase kind: phases per step and average microseconds per phase
            self.phases = {k: {"per_step": c // reps, "avg_us": 1e3 * t / c} for k, (c, t) in ph.items()}
            return sum(ts) / len(ts)
        tot, n = 0.0, 0
        for _ in range(reps):
            agg, _ = self.m.profile_step(self.rows)
            for name in self.family:
                c, t = agg.get(name, (0, 0.0))
                tot += t
                n += c
        if n != reps * self.family_launches:
            raise RuntimeError(f"step profiler saw {n} family launches, expected {reps * self.family_launches}")
        return tot / n

    def cpu(self, seconds, rows=None):
        return cpu_decode_tokps(self.L, self.C, self.V, seconds, rows or self.rows, self.base)


class StateTune29B:
    """Config 5 on the WKV-7 path: the per-layer initial states of x070 2.9B
    (L=32, H=40) trained by WKVStateTuner, `rows` 4096-token sequences per GPU
    (data-parallel, weak scaling; the tuner's NCCL allreduce under torchrun)."""
    name = "statetune"
    unit = "tok/s"
    L, H, T, N = 32, 40, 4096, 64
    NSETS = 4   # distinct per-layer input sets (each 294 MB > L2), cycled over the layers

    def __init__(self, rows=1):
        self.B = rows
        self.metric = ("x070 2.9B state-tuning tok/s on the WKV-7 path (config 5: L=32 H=40 T=4096, "
                       f"{rows} sequence/GPU; per layer train forward + checkpointed backward, "
                       "NCCL allreduce of the state gradients, global-norm clip + AdamW; chunked DPLR kernels)")

    def setup(self, torch, dev):
        from swiftrwkv_b200.state_tune import StateTuneConfig, WKVStateTuner
        self.torch = torch
        rank = torch.distributed.get_rank() if torch.distributed.is_initialized() else 0
        g = torch.Generator(device=dev)
        g.manual_seed(SEED + rank)
        shape = (self.B, self.T, self.H, self.N)
        n = lambda: torch.randn(shape, generator=g, device=dev)
        self.sets = []
        for _ in range(self.NSETS):
            r, k, v = n(), n(), n()
            w = torch.exp(-torch.exp(-torch.nn.functional.softplus(-n()) - 0.5))
            kk = torch.nn.functional.normalize(n(), dim=-1)
            b = kk * torch.sigmoid(n())
            self.sets.append([r, w, k, v, -kk, b, n()])
        self.layers = [self.sets[l % self.NSETS] for l in range(self.L)]
        self.pin = [[x.cpu().pin_memory() for x in s] for s in self.sets]
        self.tuner = WKVStateTuner(self.L, self.H, config=StateTuneConfig(), device=dev)
        self.pin_norm = torch.zeros((), dtype=torch.float32).pin_memory()
        BTHN = self.B * self.T * self.H * self.N
        BHN2 = self.B * self.H * self.N * self.N
        # canonical WKV bytes per layer: forward 4(7 BTHN + 2 BHN^2), backward 4(14 BTHN + 3 BHN^2)
        self.alg_bytes = self.L * 4 * (21 * BTHN + 5 * BHN2)
        self.bwd_bytes = 4 * (14 * BTHN + 3 * BHN2)
        self.units_per_step = self.B * self.T
        # per layer: broadcast, train forward (prep, scan, out), backward (prep, reverse
        # scan, out), grad sum; then clip + AdamW (2)
        self.launches_per_step = 8 * self.L + 2
        self.kernel = ("one layer's state gradient: chunked train forward + chunked backward "
                       "(wkv7_chunk_{prep,scan,out}, wkv7_chunk_bwd_{prep,out}, reverse scan)")
        self.h2d = sum(x.numel() * 4 for s in self.sets for x in s)
        self.d2h = 4
        self.dh = torch.empty((self.B, self.H, self.N, self.N), device=dev)

    def step(self):
        self.tuner.step(self.layers)

    def step_e2e(self):
        for d, p in zip(self.sets, self.pin):
            for x, y in zip(d, p):
                x.copy_(y, non_blocking=True)
        norm = self.tuner.step(self.layers)
        self.pin_norm.copy_(norm, non_blocking=True)

    def dominant(self):
        ops = self.tuner.ops
        *inputs, dy = self.layers[0]
        ops.layer_grad(inputs, dy, self.tuner.params[0], self.tuner.grads[0])

    @property
    def dom_bytes(self):
        # layer_grad = train forward + backward (+ two small state kernels)
        return self.alg_bytes / self.L

    def cpu(self, seconds):
        from oracle import oracle as O
        rng = np.random.default_rng(SEED)
        Ts = 256
        host = config1_inputs(rng, 1, Ts, self.H, self.N)
        dy = rng.standard_normal((1, Ts, self.H, self.N)).astype(np.float32)
        st = np.zeros((self.H, self.N, self.N), np.float32)
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < seconds or n == 0:
            O.state_layer_grad(*host, dy, st)
            n += 1
        per_layer = (time.perf_counter() - t0) / n
        return Ts / (per_layer * self.L), (f"{n} oracle layer gradients at T={Ts} H=40 "
                                            "(train forward + backward), scaled to 32 layers")


_CPU_CACHE = {}


def cpu_decode_tokps(L, C, V, seconds, rows=1, base="q4"):
    """CPU oracle decode of `rows` rows at 1.5B shapes: one layer (its
    projection GEMVs on packed weights -- 4-bit affine, or the .rwkvq sb6 / sym
    GEMVs for those bases --, the low-rank branches, WKV step + tail, all over
    the rows) and the head GEMV are timed, and the step is extrapolated as L
    layers + head."""
    from oracle import oracle as O
    from oracle.x070_oracle import lora_ranks
    key = (L, C, V, base)
    if key not in _CPU_CACHE:
        rng = np.random.default_rng(SEED)
        H, F = C // 64, 4 * C
        rk = lora_ranks(C)
        _, kind, bits = Decode15B.BASES[base]

        def q(OUT, IN):
            if kind == "sb6":
                NB = IN // 32
                return ("sb6", rng.integers(0, 256, (OUT, NB * (16 + 4 * bits)), dtype=np.uint8),
                        rng.integers(0, 64, (OUT, NB * 2), dtype=np.uint8),
                        (rng.random((OUT, NB // 8 * 2)) * 1e-3).astype(np.float16).view(np.uint16), OUT, IN, bits)
            if kind == "sym":
                return ("sym", rng.integers(0, 256, OUT * IN if bits == 8 else OUT * IN // 32 * 24, dtype=np.uint8),
                        rng.integers(0, 128, OUT * IN // 16, dtype=np.uint8),
                        (rng.random(OUT * (IN // 256)) * 1e-4).astype(np.float16).view(np.uint16), OUT, IN, bits)
            W = (rng.standard_normal((OUT, IN)) * 0.02).astype(np.float16).astype(np.float32)
            return O.affine_quantize(W)

        mats = {n: q(*sh) for n, sh in (("r", (C, C)), ("k", (C, C)), ("v", (C, C)), ("o", (C, C)),
                                         ("key", (F, C)), ("value", (C, F)))}
        lora = {n: ((rng.standard_normal((rk[n], C)) * 0.05).astype(np.float32),
                    (rng.standard_normal((C, rk[n])) * 0.05).astype(np.float32)) for n in "wavg"}
        _CPU_CACHE[key] = (C, H, mats, lora, q(V, C))
    C, H, mats, lora, head = _CPU_CACHE[key]
    rng = np.random.default_rng(SEED + rows)
    state = np.zeros((rows, H, 64, 64), np.float32)
    x = rng.standard_normal((rows, C)).astype(np.float32)
    return _cpu_decode_time(L, seconds, C, H, mats, lora, state, x, head, rows)


def _cpu_gemv(x, m):
    """One projection on the oracle: 4-bit affine (wq, scales, biases) or a
    .rwkvq ("sb6" | "sym", codes, scales, d, OUT, IN, bits) matrix."""
    from oracle import oracle as O
    kind = m[0] if isinstance(m[0], str) else "q4"
    if kind == "sb6":
        return np.stack([O.sb6_gemv(xr, *m[1:]) for xr in np.atleast_2d(x)])
    if kind == "sym":
        return O.sym_gemv(np.atleast_2d(x), *m[1:])
    return O.affine_gemv(x, *m)


def _cpu_decode_time(L, seconds, C, H, mats, lora, state, x, head, rows):
    from oracle import oracle as O
    ones, zeros = np.ones(C, np.float32), np.zeros(C, np.float32)

    def layer():
        rr = _cpu_gemv(x, mats["r"])
        kk = _cpu_gemv(x, mats["k"])
        vv = _cpu_gemv(x, mats["v"])
        hs = {n: (x @ lora[n][0].T) @ lora[n][1].T for n in "wavg"}
        wd = np.exp(-0.606531 / (1 + np.exp(-hs["w"]))).astype(np.float32)
        y, _ = O.wkv7_step(*(t.reshape(rows, H, 64) for t in (rr, wd, kk, vv, -kk, kk)), state)
        t = O.wkv_tail(y.reshape(rows, C), rr, kk, vv, ones, ones, zeros, hs["g"].astype(np.float32), H, 64)
        o = _cpu_gemv(t, mats["o"])
        hk = np.maximum(_cpu_gemv(x + o, mats["key"]), 0)
        return _cpu_gemv(hk * hk, mats["value"])

    layer()  # untimed: first-touch of the packed matrices, thread-pool start
    t0 = time.perf_counter()
    n = 0
    while time.perf_counter() - t0 < seconds / 2 or n == 0:
        layer()
        n += 1
    t_layer = (time.perf_counter() - t0) / n
    t0 = time.perf_counter()
    m = 0
    while time.perf_counter() - t0 < seconds / 4 or m == 0:
        _cpu_gemv(x, head)
        m += 1
    t_head = (time.perf_counter() - t0) / m
    return rows / (L * t_layer + t_head), (f"{rows} rows; {n} timed x070 1.5B layers + {m} head GEMVs "
                                           f"over all rows, step = {L} layers + head")


def cpu_threads(cores):
    return {"openmp": cores, "blas": int(os.environ.get("OPENBLAS_NUM_THREADS", BLAS_THREADS))}


class RwkvqGemvSuite:
    """Config 2's .rwkvq variant: the sb6 (5-bit: 4 + 1 bit-plane) and sym (6-
    and 8-bit) GEMVs at the 1.5B projection shapes (2048x2048, 8192x2048,
    2048x8192, 65536x2048), fp16 activations, through rwkv_sb6_gemv /
    rwkv_sym_gemv (RwkvqSb6GEMV.swift:69-208, RwkvqSymGEMV.swift:89-263).
    Synthetic codes and scales (values do not change the timing)."""
    name = "gemv_rwkvq"
    unit = "GB/s"
    MATS = [(2048, 2048), (8192, 2048), (2048, 8192), (65536, 2048)]
    FMTS = [("sb6", 1), ("sym", 6), ("sym", 8)]

    def __init__(self, rows=1):
        self.rows = rows
        self.metric = (f".rwkvq GEMV GB/s (config 2: sb6 5-bit, sym 6 / 8-bit at the 1.5B projection shapes, "
                       f"rows {rows}, fp16 x)")

    @staticmethod
    def wbytes(kind, bits, OUT, IN):
        if kind == "sb6":
            return OUT * IN * (16 + 4 * bits + 2) // 32 + OUT * IN // 256 * 4
        code = OUT * IN if bits == 8 else OUT * IN * 24 // 32
        return code + OUT * IN // 16 + OUT * IN // 256 * 2

    def setup(self, torch, dev):
        from swiftrwkv_b200 import _lib
        self.torch, self._lib = torch, _lib
        g = torch.Generator(device=dev).manual_seed(SEED)
        R = self.rows
        u8 = lambda n: torch.randint(0, 256, (n,), generator=g, device=dev, dtype=torch.int32).to(torch.uint8)
        self.jobs = []
        for kind, bits in self.FMTS:
            for OUT, IN in self.MATS:
                if kind == "sb6":
                    NB = IN // 32
                    qblk = u8(OUT * NB * (16 + 4 * bits))
                    q2 = u8(OUT * NB * 2) & 0x3F          # qs < 64, qm small and positive (valid int8)
                    d = (torch.rand(OUT * (NB // 8) * 2, generator=g, device=dev) * 1e-3).half()
                else:
                    qblk = u8(OUT * IN if bits == 8 else OUT * IN // 32 * 24)
                    q2 = u8(OUT * IN // 16) & 0x7F
                    d = (torch.rand(OUT * (IN // 256), generator=g, device=dev) * 1e-4).half()
                x = torch.randn((R, IN), generator=g, device=dev).half()
                y = torch.empty((R, OUT), device=dev, dtype=torch.float32)
                self.jobs.append((kind, bits, OUT, IN, qblk, q2, d, x, y))
        mb = lambda kind, bits, OUT, IN: self.wbytes(kind, bits, OUT, IN) + R * IN * 2 + R * OUT * 4
        self.alg_bytes = sum(mb(j[0], j[1], j[2], j[3]) for j in self.jobs)
        self.units_per_step = self.alg_bytes / 1e9
        self.launches_per_step = len(self.jobs) * ((R + 3) // 4)
        self.dom = self.jobs[-1]  # sym 8-bit head
        self.dom_bytes = mb(*self.dom[:4])
        self.kernel = "sym_gemv_tile_kernel (8-bit), 65536x2048"
        self.h2d = sum(R * j[3] * 2 for j in self.jobs)
        self.d2h = sum(R * j[2] * 4 for j in self.jobs)
        self.pin_x = [torch.empty((R, j[3]), dtype=torch.float16).pin_memory() for j in self.jobs]
        self.pin_y = [torch.empty((R, j[2]), dtype=torch.float32).pin_memory() for j in self.jobs]

    def _gemv(self, kind, bits, OUT, IN, qblk, q2, d, x, y):
        _lib, P = self._lib, self._lib.P
        st = P(self.torch.cuda.current_stream().cuda_stream)
        if kind == "sb6":
            _lib.call("rwkv_sb6_gemv", 2, P(x.data_ptr()), P(qblk.data_ptr()), P(q2.data_ptr()), P(d.data_ptr()),
                      P(y.data_ptr()), self.rows, OUT, IN, bits, st)
        else:
            _lib.call("rwkv_sym_gemv", 2, P(x.data_ptr()), P(qblk.data_ptr()), P(q2.data_ptr()), P(d.data_ptr()),
                      P(y.data_ptr()), self.rows, OUT, IN, bits, OUT, st)

    def step(self):
        for j in self.jobs:
            self._gemv(*j)

    def dominant(self):
        self._gemv(*self.dom)

    def step_e2e(self):
        for j, px in zip(self.jobs, self.pin_x):
            j[7].copy_(px, non_blocking=True)
        self.step()
        for j, py in zip(self.jobs, self.pin_y):
            py.copy_(j[8], non_blocking=True)

    def cpu(self, seconds):
        """The oracle's sb6 GEMV (RwkvqSb6GEMV.swift:103-145 order) on one
        2048 x 2048 matrix, one row."""
        from oracle import oracle as O
        rng = np.random.default_rng(SEED)
        OUT, IN, xb = 2048, 2048, 1
        NB = IN // 32
        qblk = rng.integers(0, 256, (OUT, NB * (16 + 4 * xb)), dtype=np.uint8)
        qsqm = (rng.integers(0, 64, (OUT, NB * 2))).astype(np.uint8)
        ddm = (np.abs(rng.standard_normal((OUT, NB // 8 * 2))) * 1e-3).astype(np.float16).view(np.uint16)
        x = rng.standard_normal((IN,)).astype(np.float32)
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < seconds or n == 0:
            O.sb6_gemv(x, qblk, qsqm, ddm, OUT, IN, xb)
            n += 1
        dt = time.perf_counter() - t0
        return n * self.wbytes("sb6", xb, OUT, IN) / dt / 1e9, f"{n} sb6 GEMVs of 2048x2048 (5-bit), 1 row"


class ProjBackward29B:
    """The frozen-base projection backward dX = bf16(bf16(dY) W_bf16) (the
    bf16 VJP of X070Backbone.baseMatmul, X070Backbone.swift:337-356) over one
    layer of config 5's frozen bf16 2.9B base at 4096 tokens per GPU: the four
    C x C projections (r, k, v, o), key (4C x C) and value (C x 4C), through
    rwkv_gemm_dx.  Tensor-bound: the roofline is the measured bf16 peak."""
    name = "dx"
    unit = "TFLOP/s"
    bound = "tensor"
    C, TOK = 2560, 4096

    def __init__(self):
        self.metric = ("projection backward TFLOP/s (config 5: frozen bf16 2.9B base, one layer's dX = dY W "
                       "for r/k/v/o, key, value at 4096 tokens, tcgen05)")

    def setup(self, torch, dev):
        from swiftrwkv_b200 import _lib
        self.torch, self._lib = torch, _lib
        C, F, T = self.C, 4 * self.C, self.TOK
        self.shapes = [(C, C)] * 4 + [(F, C), (C, F)]  # (OUT, IN) of the forward projection
        g = torch.Generator(device="cpu").manual_seed(SEED)
        self.mats = []
        for OUT, IN in self.shapes:
            W = (torch.randn((OUT, IN), generator=g) * 0.02).to(torch.bfloat16).to(dev)
            dy = torch.randn((T, OUT), generator=g).to(torch.bfloat16).to(dev)
            dx = torch.empty((T, IN), device=dev, dtype=torch.float32)
            self.mats.append((OUT, IN, W, dy, dx))
        fl = lambda OUT, IN: 2.0 * T * OUT * IN
        self.flops = sum(fl(o, i) for o, i in self.shapes)
        self.alg_bytes = sum(o * i * 2 + T * o * 2 + T * i * 4 for o, i in self.shapes)
        self.units_per_step = self.flops / 1e12
        self.launches_per_step = len(self.shapes)
        self.dom_flops = fl(*self.shapes[4])  # the key matrix's backward
        self.kernel = "gemm_dx_kernel<DX_BF16, 256> (tcgen05, A = W^T MN-major via TMA), 4096 x 10240 -> 2560"
        self.h2d = sum(T * o * 2 for o, _ in self.shapes)
        self.d2h = sum(T * i * 4 for _, i in self.shapes)
        self.pin_dy = [torch.empty((T, o), dtype=torch.bfloat16).pin_memory() for o, _ in self.shapes]
        self.pin_dx = [torch.empty((T, i), dtype=torch.float32).pin_memory() for _, i in self.shapes]

    def _dx(self, OUT, IN, W, dy, dx):
        _lib, P = self._lib, self._lib.P
        st = P(self.torch.cuda.current_stream().cuda_stream)
        _lib.call("rwkv_gemm_dx", 1, P(dy.data_ptr()), 1, P(W.data_ptr()), 0, P(dx.data_ptr()), self.TOK, OUT, IN, 0, st)

    def step(self):
        for m in self.mats:
            self._dx(*m)

    def dominant(self):
        self._dx(*self.mats[4])

    def step_e2e(self):
        for m, pd in zip(self.mats, self.pin_dy):
            m[3].copy_(pd, non_blocking=True)
        self.step()
        for m, px in zip(self.mats, self.pin_dx):
            px.copy_(m[4], non_blocking=True)

    def cpu(self, seconds):
        """The oracle's restatement (numpy float64 matmul of the bf16 operands,
        one BLAS thread) on 256-token slices of the C x C shape."""
        from oracle import oracle as O
        rng = np.random.default_rng(SEED)
        C, T = self.C, 256
        dy = rng.standard_normal((T, C)).astype(np.float32)
        W = (rng.standard_normal((C, C)) * 0.02).astype(np.float32)
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < seconds or n == 0:
            O.base_matmul_vjp(dy, W)
            n += 1
        dt = time.perf_counter() - t0
        self.cpu_cores = 1
        return n * 2.0 * T * C * C / dt / 1e12, f"{n} backward products of {T} tokens x {C} x {C}"


WORKLOADS = {"decode": Decode15B, "wkv7": WKV7Prefill, "wkv7train": WKV7Train, "gemv": GemvSuite,
             "statetune": StateTune29B, "dx": ProjBackward29B,
             "gemv_rwkvq": RwkvqGemvSuite}


# ----------------------------------------------------------------------- timing

def timed(torch, fn, steps, warmup, flush, dist):
    for _ in range(warmup):
        flush()
        fn()
    torch.cuda.synchronize()
    if dist:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    evs = []
    for _ in range(steps):
        flush()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        evs.append((s, e))
    torch.cuda.synchronize()
    if dist:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in evs]


def max_over_ranks(torch, val, dist):
    if not dist:
        return val
    t = torch.tensor([val], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def run_reference(args, rank):
    """CPU arm: the oracle restatement on all host cores, same metric/config.
    Under torchrun rank 0 alone runs it, over the whole job's rows."""
    if rank != 0:
        return
    from oracle import oracle as O
    O.build()
    cores = os.cpu_count() or 1
    O.set_threads(cores)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    wl = make_workload(args)
    if wl.name in ("wkv7", "wkv7train"):
        rng = np.random.default_rng(SEED)
        wl.host = config1_inputs(rng)
        if wl.name == "wkv7train":
            wl.host.append(rng.standard_normal(wl.host[0].shape).astype(np.float32))
    per = []
    sample = ""
    # each step a bounded sample: the whole run stays within a few minutes
    budget = min(4.0, 120.0 / (args.warmup + args.steps))
    config = {"workload": wl.name}
    for i in range(args.warmup + args.steps):
        if wl.name == "decode":
            v, sample = wl.cpu(budget, rows=wl.rows * world)
        else:
            v, sample = wl.cpu(budget)
        if i >= args.warmup:
            per.append(v)
    if wl.name == "decode":
        config.update({"model": "x070 1.5B (L=24 C=2048 H=32 V=65536 FFN=8192)", "rows_per_gpu": wl.rows,
                       "global_batch": wl.rows * world, "base": wl.base_label})
    value = statistics.median(per)
    out = {"impl": "reference", "metric": wl.metric, "value": value, "unit": wl.unit,
           "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
           "higher_is_better": True, "dtype": "f32", "data": "synthetic",
           "config": config,
           "cpu_baseline": {"value": value, "unit": wl.unit, "cores": getattr(wl, "cpu_cores", cores), "kind": "port",
                            "threads": cpu_threads(getattr(wl, "cpu_cores", cores)), "sample": sample},
           "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(out))


def wkv_prefill_line(torch, dev, args, peaks, flush_l2):
    """BASELINE's second metric beside decode: WKV-7 prefill tok/s on config 1
    (the chunked forward), with its own roofline; timed like the main line."""
    pw = WKV7Prefill()
    pw.setup(torch, dev)
    times = timed(torch, pw.step, args.steps, args.warmup, flush_l2, False)
    e2e = timed(torch, pw.step_e2e, args.steps, args.warmup, flush_l2, False)
    ms = sum(times) / len(times)
    ms_e2e = sum(e2e) / len(e2e)
    gbs = pw.alg_bytes / (ms / 1e3) / 1e9
    return {"metric": pw.metric, "value": pw.units_per_step / (ms / 1e3), "unit": pw.unit,
            "ms_per_step": ms, "dtype": "f32", "l2": "flushed (256 MB write) before every timed step",
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / peaks["hbm_gbs"], "traffic": None, "peak_src": peaks["src"],
                         "kernel": "wkv7_chunk_{prep,scan,out}: the three-launch step (canonical bytes "
                                   "4(7 BTHN + BHN^2) over the step's time)",
                         "kernel_ms": ms},
            "e2e": {"value": pw.units_per_step / (ms_e2e / 1e3), "unit": pw.unit,
                    "h2d_bytes_per_step": pw.h2d, "d2h_bytes_per_step": pw.d2h},
            "gpu_launches": pw.launches_per_step * args.steps, "_wl": pw}


def config3_line(torch, dev, args, peaks):
    """random-init x070 0.1B (L=12, C=768, H=12, vocab
    65536) over a dense bf16 base with bf16 activations; a 1024-token prefill
    (uniform ids) at batch 1, then 256 greedy decode steps.  Weights (0.19 GB)
    exceed L2 only with the head; timed as the workload runs (no flush)."""
    from swiftrwkv_b200.x070 import X070Backbone, X070Config
    L, C, V, T, NEW = 12, 768, 65536, 1024, 256
    m = X070Backbone(X070Config(L, C, V), max_rows=1, act="bf16", base="bf16").init_random(seed=SEED)
    rng = np.random.default_rng(SEED + 3)
    prompt = rng.integers(0, V, (1, T), dtype=np.int32)
    dprompt = torch.from_numpy(prompt).to(dev)
    st = torch.cuda.current_stream()
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def prefill():
        m.reset(1)
        m.prefill(dprompt, logits=False)

    def decode():
        for _ in range(NEW):
            m.step_greedy(1, None, use_graph=True)

    for _ in range(max(args.warmup, 3)):
        prefill()
        decode()
    torch.cuda.synchronize()
    pf, dc = [], []
    for _ in range(max(3, min(args.steps, 10))):
        a, b, c = ev(), ev(), ev()
        a.record(st)
        prefill()
        b.record(st)
        decode()
        c.record(st)
        torch.cuda.synchronize()
        pf.append(a.elapsed_time(b))
        dc.append(b.elapsed_time(c))
    pf_ms, dc_ms = statistics.median(pf), statistics.median(dc)
    # end to end through generate (host prompt in, host tokens out, per-token sync)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    m.reset(1)
    out = m.generateBatch(prompt, NEW)
    e2e_s = time.perf_counter() - t0
    H = C // 64
    step_bytes = m.weight_bytes + L * H * 64 * 64 * 4 * 2 + L * C * 4 * 2 * 2
    gbs = step_bytes / (dc_ms / NEW / 1e3) / 1e9
    m.close()
    return {"metric": "x070 0.1B bf16 (config 3): 1024-token prefill tok/s and greedy decode tok/s, batch 1",
            "prefill_tok_s": T / (pf_ms / 1e3), "prefill_ms": pf_ms,
            "decode_tok_s": NEW / (dc_ms / 1e3), "decode_ms_per_token": dc_ms / NEW,
            "dtype": "bf16", "data": "synthetic (random init, uniform ids)",
            "decode_roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                "frac": gbs / peaks["hbm_gbs"], "alg_bytes_per_token": step_bytes,
                                "peak_src": peaks["src"]},
            "e2e": {"value": (T + NEW) / e2e_s, "unit": "tok/s (prompt + generated, wall clock, generate API)",
                    "tokens_out": int(out.size)}}


def make_workload(args):
    if args.workload == "decode":
        return Decode15B(args.rows or 64, args.prompt, args.decode_path, args.base)
    if args.workload == "gemv":
        return GemvSuite(args.rows or 1)
    if args.workload == "gemv_rwkvq":
        return RwkvqGemvSuite(args.rows or 1)
    if args.workload == "statetune":
        return StateTune29B(args.rows or 1)
    return WORKLOADS[args.workload]()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="decode", choices=sorted(WORKLOADS))
    ap.add_argument("--rows", type=int, default=None,
                    help="decode rows per GPU (default 64) / GEMV activation rows (default 1)")
    ap.add_argument("--prompt", type=int, default=128, help="decode prompt tokens per row")
    ap.add_argument("--decode-path", default="launches", choices=["launches", "persistent"],
                    help="decode: one graph of per-op launches (default) or the persistent one-launch step "
                         "(9..64 rows, fp16 activations, 4-bit base)")
    ap.add_argument("--base", default="q4", choices=sorted(Decode15B.BASES),
                    help="decode: the projection / head container (q4: MLX affine 4-bit g64, default; "
                         "sb6 / sym6 / sym8: native .rwkvq matrices)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank)

    import torch
    dist = world > 1
    torch.cuda.set_device(local)
    if dist:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    from swiftrwkv_b200 import _lib
    _lib.lib()

    wl = make_workload(args)
    wl.setup(torch, dev)
    flush_buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_l2 = lambda: flush_buf.zero_()
    step_flush = (lambda: None) if wl.name == "decode" else flush_l2
    l2_note = ("inputs larger than L2 (weights 0.86 GB + state per step); no flush"
               if wl.name == "decode" else "flushed (256 MB write) before every timed step")

    clk = ClockSampler(local)
    clk.start()
    times = timed(torch, wl.step, args.steps, args.warmup, step_flush, dist)
    clocks = clk.stop()
    e2e_times = timed(torch, wl.step_e2e, args.steps, args.warmup, step_flush, dist)

    ms = max_over_ranks(torch, sum(times) / len(times), dist)
    ms_e2e = max_over_ranks(torch, sum(e2e_times) / len(e2e_times), dist)
    units = wl.units_per_step * world
    value = units / (ms / 1e3)
    e2e_value = units / (ms_e2e / 1e3)
    peaks = load_peaks()
    local_ms = sum(times) / len(times)
    step_gbs = wl.alg_bytes / (local_ms / 1e3) / 1e9
    if hasattr(wl, "dominant_ms"):
        # the dominant kernel family timed inside the step (per-launch device times)
        dom_ms = wl.dominant_ms(3)
        achieved = wl.dom_bytes / (dom_ms / 1e3) / 1e9
        kernel = wl.kernel
    elif hasattr(wl, "dominant"):
        # the dominant kernel timed on its own stream position, L2 flushed before each launch
        dt = timed(torch, wl.dominant, args.steps, args.warmup, flush_l2, False)
        dom_ms = sum(dt) / len(dt)
        if getattr(wl, "bound", "hbm") == "tensor":
            achieved = wl.dom_flops / (dom_ms / 1e3) / 1e12
        else:
            achieved = wl.dom_bytes / (dom_ms / 1e3) / 1e9
        kernel = wl.kernel
    else:
        dom_ms = local_ms / wl.launches_per_step
        achieved = wl.alg_bytes / wl.launches_per_step / (dom_ms / 1e3) / 1e9
        kernel = wl.kernel
    result = {
        "metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": ("f32" if wl.name in ("wkv7", "wkv7train", "statetune") else
                  "sb6 u5 / sym u6, i8 x f16 -> f32" if wl.name == "gemv_rwkvq" else "u4 x f16 -> f32"),
        "data": "synthetic",
        "config": {"workload": wl.name, "l2": l2_note, "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                     # the committed captures cover the per-op launches, not the persistent step
                     "traffic": None if getattr(wl, "persistent", False) else measured_traffic(wl),
                     "peak_src": peaks["src"], "kernel": kernel, "kernel_ms": dom_ms},
        "step_roofline": {"alg_bytes": wl.alg_bytes, "achieved": step_gbs,
                          "frac": step_gbs / peaks["hbm_gbs"], "unit": "GB/s"},
        "e2e": {"value": e2e_value, "unit": wl.unit, "h2d_bytes_per_step": wl.h2d,
                "d2h_bytes_per_step": wl.d2h},
        "gpu_launches": wl.launches_per_step * args.steps,
        "clocks": clocks,
    }
    if getattr(wl, "bound", "hbm") == "tensor":
        # a contraction: FLOPs against the measured dense bf16 peak (burst: the kernel is timed alone)
        step_tf = wl.flops / (local_ms / 1e3) / 1e12
        result["roofline"].update({"bound": "tensor", "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                                   "frac": achieved / peaks["bf16_tflops"], "traffic": None})
        result["step_roofline"] = {"flops": wl.flops, "achieved": step_tf, "frac": step_tf / peaks["bf16_tflops"],
                                   "unit": "TFLOP/s"}
        result["dtype"] = "bf16 x bf16 -> f32 (bf16-rounded)"
        result["config"].update({"model": "x070 2.9B frozen bf16 base (C=2560, FFN 10240), one layer",
                                 "tokens_per_gpu": wl.TOK})
    if wl.name == "statetune":
        result["config"].update({"model": "x070 2.9B WKV path (L=32 H=40 N=64)", "seq_len": wl.T,
                                 "rows_per_gpu": wl.B, "global_batch": wl.B * world,
                                 "parallelism": f"dp{world} (NCCL allreduce of state gradients)",
                                 "inputs": f"{wl.NSETS} distinct per-layer sets cycled over 32 layers"})
    if getattr(wl, "phases", None):
        result["roofline"]["phases"] = wl.phases
    if wl.name == "decode":
        result["config"]["decode_path"] = "persistent" if wl.persistent else "launches"
        result["config"].update({"model": "x070 1.5B (L=24 C=2048 H=32 V=65536 FFN=8192)",
                                 "rows_per_gpu": wl.rows, "global_batch": wl.rows * world,
                                 "prompt": wl.PROMPT, "base": wl.base_label})
    if wl.name == "decode" and world == 1:
        result["prefill"] = wkv_prefill_line(torch, dev, args, peaks, flush_l2)
        result["config3"] = config3_line(torch, dev, args, peaks)
    if rank == 0 and world == 1:
        from oracle import oracle as O
        O.build()
        cores = os.cpu_count() or 1
        O.set_threads(cores)
        v, sample = wl.cpu(args.cpu_seconds)
        used = getattr(wl, "cpu_cores", cores)
        result["cpu_baseline"] = {"value": v, "unit": wl.unit, "cores": used, "kind": "port",
                                  "threads": cpu_threads(used), "sample": sample}
        if "prefill" in result:
            pw = result["prefill"].pop("_wl")
            pv, psample = pw.cpu(min(args.cpu_seconds, 5.0))
            result["prefill"]["cpu_baseline"] = {"value": pv, "unit": pw.unit, "cores": cores, "kind": "port",
                                                 "threads": cpu_threads(cores), "sample": psample}
    if rank == 0:
        print(json.dumps(result))
    if dist:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
