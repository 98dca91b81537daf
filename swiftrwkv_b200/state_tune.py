"""Data-parallel state tuning over the WKV-7 path.

The trainable parameters are every layer's initial WKV state [H, N, N] fp32,
shared by all sequences of the batch (StateTrainableSet,
Sources/RWKVGen/InitialState.swift:176-251, `train: [.wkv]`).  One step:

  for each layer, top to bottom (SequentialBackward.swift:180-219 order):
      h_in = broadcast(state[l])                     rwkv_state_broadcast
      train forward with 16-token checkpoints        rwkv_wkv7_train_forward_chunked
      backward from the layer's upstream dy          rwkv_wkv7_backward_chunked
      grad[l] = sum over the local batch of dh_in    rwkv_state_grad_sum
      allreduce(sum) of grad[l] over the ranks, started as soon as the
      layer is done (NCCL, asynchronous, one bucket per layer)
  wait for the allreduces; average (x 1/world), clip by global norm, AdamW
                                                     rwkv_adamw_clip_step

which is Trainer.run's step (Sources/RWKVGen/Training/Trainer.swift:141-161)
with the data-parallel sum in place of gradient accumulation.  The per-layer
WKV inputs (r, w, k, v, a, b) and upstream gradients dy are given: the
backbone that produces them (projections, norms, the loss) is not part of the
WKV path.  Each rank takes its own contiguous slice of the batch; after the
allreduce every rank holds the same gradient and makes the same update, so
the states stay identical without a broadcast.

All arithmetic runs in librwkvcuda (no CPU fallback); torch supplies device
memory, the stream and torch.distributed.  `ops` exists so that the rank
logic can run against another implementation of the same five operations.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import call

WKV7_HEAD_SIZE = 64
WKV7_CHUNK = 16

_DT = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}


@dataclass
class StateTuneConfig:
    """The optimizer fields of StateTuneConfig (InitialState.swift:253-318),
    with its defaults."""
    lr: float = 3e-4
    lrMin: float = 3e-5
    schedule: str = "cosine"   # LRSchedule: "constant" | "cosine" | "linear"
    warmupSteps: int = 10
    maxSteps: int = 500
    gradClip: float = 1.0      # <= 0: no clipping (the norm is still reported)
    beta1: float = 0.9
    beta2: float = 0.99
    adamEps: float = 1e-8
    weightDecay: float = 0.0

    def __post_init__(self):
        if self.schedule not in ("constant", "cosine", "linear"):
            raise ValueError(f"schedule {self.schedule!r}: constant, cosine or linear")

    def learningRate(self, step: int) -> float:
        """TrainingConfig.learningRate(at:) (TrainingConfig.swift:83-98), in
        fp32 like the reference's Float arithmetic."""
        f = np.float32
        lr, lr_min = f(self.lr), f(self.lrMin)
        if self.warmupSteps > 0 and step < self.warmupSteps:
            return float(lr * f(step + 1) / f(self.warmupSteps))
        if self.schedule == "constant":
            return float(lr)
        denom = max(1, self.maxSteps - self.warmupSteps)
        progress = min(f(step - self.warmupSteps) / f(denom), f(1.0))
        if self.schedule == "cosine":
            decay = f(0.5) * (f(1.0) + np.cos(f(math.pi) * f(progress), dtype=np.float32))
        else:
            decay = f(1.0) - f(progress)
        return float(lr_min + (lr - lr_min) * f(decay))

    def bias_corrections(self, t: int) -> tuple[float, float]:
        """c1 = 1 - beta1^t, c2 = 1 - beta2^t as Trainer.swift:151-153 forms
        them: the power in double of the fp32 beta, then fp32."""
        f = np.float32
        c1 = f(1) - f(math.pow(float(f(self.beta1)), float(t)))
        c2 = f(1) - f(math.pow(float(f(self.beta2)), float(t)))
        return float(c1), float(c2)


def _p(t):
    return None if t is None else _lib.P(t.data_ptr())


def _stream():
    return _lib.P(torch.cuda.current_stream().cuda_stream)


class CudaStateOps:
    """The five device operations of a state-tuning step, through the C ABI.
    Scratch buffers are allocated once per shape and reused."""

    def __init__(self):
        self._seq: dict = {}
        self._adam: dict = {}

    def _buffers(self, like: torch.Tensor):
        B, T, H, N = like.shape
        key = (B, T, H, N, like.dtype, like.device)
        s = self._seq.get(key)
        if s is None:
            dev = like.device
            ws_bytes = max(int(_lib.lib().rwkv_wkv7_backward_chunked_workspace_size(B, T, H, N)),
                           int(_lib.lib().rwkv_wkv7_forward_chunked_workspace_size(B, T, H, N)))
            s = {
                "h_in": torch.empty((B, H, N, N), device=dev, dtype=torch.float32),
                "y": torch.empty_like(like),
                "ck": torch.empty((B, H, T // WKV7_CHUNK, N, N), device=dev, dtype=torch.float32),
                "d": [torch.empty_like(like) for _ in range(6)],
                "dh_in": torch.empty((B, H, N, N), device=dev, dtype=torch.float32),
                "ws": torch.empty(max(ws_bytes, 16), device=dev, dtype=torch.uint8),
                "ws_bytes": ws_bytes,
            }
            self._seq = {key: s}  # one live shape at a time
        return s

    def layer_grad(self, inputs, dy, state, grad):
        """grad [H,N,N] = sum over the batch of d(sum y*dy)/d h_in with
        h_in[b] = state for every b; inputs r..b and dy [B,T,H,N]."""
        r, w, k, v, a, b = inputs
        B, T, H, N = r.shape
        s = self._buffers(r)
        st = _stream()
        dt = _DT[r.dtype]
        call("rwkv_state_broadcast", _p(state), _p(s["h_in"]), B, H, N, st)
        call("rwkv_wkv7_train_forward_chunked", dt, *map(_p, inputs), _p(s["h_in"]), _p(s["y"]), None,
             None, _p(s["ck"]), B, T, H, N, _p(s["ws"]), s["ws_bytes"], st)
        call("rwkv_wkv7_backward_chunked", dt, *map(_p, inputs), _p(s["h_in"]), _p(s["ck"]), _p(dy), None,
             *map(_p, s["d"]), _p(s["dh_in"]), B, T, H, N, _p(s["ws"]), s["ws_bytes"], st)
        call("rwkv_state_grad_sum", _p(s["dh_in"]), _p(grad), B, H, N, 0, st)

    def adamw(self, param, m, v, grad, norm_out, *, grad_scale, clip, lr, beta1, beta2, eps,
              weight_decay, c1, c2):
        n = param.numel()
        ws_bytes = int(_lib.lib().rwkv_adamw_workspace_size(n))
        ws = self._adam.get((n, param.device))
        if ws is None:
            ws = torch.empty(max(ws_bytes, 16), device=param.device, dtype=torch.uint8)
            self._adam = {(n, param.device): ws}
        call("rwkv_adamw_clip_step", _p(param), _p(m), _p(v), _p(grad), n, grad_scale, clip, lr,
             beta1, beta2, eps, weight_decay, c1, c2, _p(norm_out), _p(ws), ws_bytes, _stream())


class WKVStateTuner:
    """State tuning of `n_layer` initial WKV states [H, N, N] over the WKV-7
    path, data-parallel over the ranks of `group` (None: the default process
    group when torch.distributed is initialised, else a single process).

    step(layers) takes, for this rank's slice of the batch, one tuple
    (r, w, k, v, a, b, dy) of [B_local, T, H, N] tensors per layer, T % 16 == 0,
    and returns the global gradient norm as a device tensor (before
    clipping, as Trainer reports it)."""

    def __init__(self, n_layer: int, n_head: int, head_size: int = WKV7_HEAD_SIZE,
                 config: StateTuneConfig | None = None, initial: torch.Tensor | None = None,
                 device=None, group=None, ops=None, grad_scale: float | None = None):
        if head_size != WKV7_HEAD_SIZE:
            raise ValueError(f"head_size {head_size}: the WKV-7 kernels take {WKV7_HEAD_SIZE}")
        self.cfg = config or StateTuneConfig()
        self.L, self.H, self.N = n_layer, n_head, head_size
        self.device = torch.device(device) if device is not None else (
            initial.device if initial is not None else torch.device("cuda"))
        shape = (n_layer, n_head, head_size, head_size)
        if initial is not None:
            if tuple(initial.shape) != shape:
                raise ValueError(f"initial {tuple(initial.shape)} must be {list(shape)}")
            self.params = initial.to(self.device, torch.float32).clone().contiguous()
        else:
            self.params = torch.zeros(shape, device=self.device, dtype=torch.float32)
        self.m = torch.zeros_like(self.params)
        self.v = torch.zeros_like(self.params)
        self.grads = torch.zeros_like(self.params)
        self.norm = torch.zeros((), device=self.device, dtype=torch.float32)
        self.t = 0          # optimizer steps taken (Trainer.t)
        self.step_index = 0  # schedule position (Trainer's `step`)
        self.ops = ops if ops is not None else CudaStateOps()
        self.group = group
        dist = torch.distributed
        self.world = dist.get_world_size(group) if (dist.is_available() and dist.is_initialized()) else 1
        self.grad_scale = (1.0 / self.world) if grad_scale is None else float(grad_scale)

    @staticmethod
    def local_slice(global_batch: int, rank: int, world: int) -> slice:
        """This rank's contiguous share of a global batch (equal shares)."""
        if global_batch % world:
            raise ValueError(f"global batch {global_batch} does not split over {world} ranks")
        per = global_batch // world
        return slice(rank * per, (rank + 1) * per)

    def _check(self, layers):
        if len(layers) != self.L:
            raise ValueError(f"{len(layers)} layers given, the tuner has {self.L}")
        for l, t in enumerate(layers):
            if len(t) != 7:
                raise ValueError(f"layer {l}: expected (r, w, k, v, a, b, dy)")
            shp = tuple(t[0].shape)
            if len(shp) != 4 or shp[2] != self.H or shp[3] != self.N:
                raise ValueError(f"layer {l}: r {shp} must be [B, T, {self.H}, {self.N}]")
            if shp[1] % WKV7_CHUNK:
                raise ValueError(f"layer {l}: T ({shp[1]}) must be a multiple of CHUNK {WKV7_CHUNK}")
            for x in t[1:]:
                if tuple(x.shape) != shp:
                    raise ValueError(f"layer {l}: every tensor must be {list(shp)}")

    def step(self, layers):
        self._check(layers)
        dist = torch.distributed
        works = []
        for l in reversed(range(self.L)):
            *inputs, dy = layers[l]
            self.ops.layer_grad(inputs, dy, self.params[l], self.grads[l])
            if self.world > 1:
                works.append(dist.all_reduce(self.grads[l], op=dist.ReduceOp.SUM, group=self.group,
                                             async_op=True))
        for w in works:
            w.wait()
        lr = self.cfg.learningRate(self.step_index)
        self.t += 1
        c1, c2 = self.cfg.bias_corrections(self.t)
        self.ops.adamw(self.params, self.m, self.v, self.grads, self.norm,
                       grad_scale=self.grad_scale, clip=self.cfg.gradClip, lr=lr,
                       beta1=self.cfg.beta1, beta2=self.cfg.beta2, eps=self.cfg.adamEps,
                       weight_decay=self.cfg.weightDecay, c1=c1, c2=c2)
        self.step_index += 1
        return self.norm

    def checkpoint(self) -> dict:
        """Parameters, Adam moments and counters (Trainer.checkpointArrays,
        Trainer.swift:203-215: param/, m/, v/ and _meta/step = [step, t])."""
        return {"param": self.params.clone(), "m": self.m.clone(), "v": self.v.clone(),
                "_meta/step": (self.step_index, self.t)}

    def restore(self, ck: dict):
        """Trainer.restore(fromCheckpoint:) (Trainer.swift:225-247)."""
        for name in ("param", "m", "v"):
            if name not in ck:
                raise KeyError(f"checkpoint has no tensor {name}/")
            if tuple(ck[name].shape) != tuple(self.params.shape):
                raise ValueError(f"{name}/ {tuple(ck[name].shape)} must be {tuple(self.params.shape)}")
        self.params.copy_(ck["param"])
        self.m.copy_(ck["m"])
        self.v.copy_(ck["v"])
        self.step_index, self.t = (int(x) for x in ck["_meta/step"])
