"""The MLP training step with its state resident on one GPU.

The same step as drift_b200.mlp (Pass and Trainer of
java/src/main/java/io/drift/train/), with the weights, the Adam moments, the
cast copies, the gradients and the delayed-scaling amax history held in device
memory across steps. Each step's boundary traffic is the tokens, the targets
and the small activations that meet Java's transcendental functions:
Math.tanh, Math.exp and Math.log are not specified to the bit, so tanh and the
softmax run on the host in double exactly as drift_b200.mlp runs them (two
B x hidden round trips and one B x vocab round trip per step). Everything else runs as engine kernels:

* the embedding lookup and its ordered gradient (Pass.java:122-126, :168-179);
* the casts (Quant.quantize), with per-tensor amax and delayed scaling
  (Pass.scaleFor, :249-271);
* the forward, dgrad and wgrad contractions (:184-241);
* the bias gradients (:234-240) and tanh's derivative (:279-283);
* the Adam update with optional FP32 masters (Trainer.java:246-269).

The results equal drift_b200.mlp's, and so the oracle's, bit for bit.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import numpy as np

from . import _lib
from .fmt import Rounding
from .kernel import (NumericPolicy, Scaling, _stream_ptr, _tptr, amax_dev, gemm_dev,
                     per_tensor_scale_dev, quantize_dev)
from .mlp import LAYERS, T_G, T_W, T_X, Net, StepRecord, compare, softmax_xent


def _call(name: str, *args) -> None:
    _lib.check(getattr(_lib.load(), name)(_lib.Context.current().handle, *args))


class DevicePass:
    """One policy's pass with its casts, history and Rng state on the GPU
    (Pass.java:26-90). Parameters are the trainer's device tensors."""

    def __init__(self, p: NumericPolicy, net: Net, params, batch: int, rng_seed: int, device):
        import torch

        self.torch = torch
        self.p = p
        self.net = net
        self.params = params  # embed, w1, b1, w2, b2, w3, b3 (device)
        self.batch = batch
        self.dev = device
        f64 = dict(dtype=torch.float64, device=device)
        self.state = torch.tensor([_signed(rng_seed)], dtype=torch.int64, device=device)
        self.clamped = torch.zeros(3, dtype=torch.int64, device=device)
        self.cast = np.zeros(3, dtype=np.int64)
        hl = max(1, p.amax_history)
        self.hist_len = hl
        self.history = torch.zeros((LAYERS, 3, hl), **f64)
        self.history_count = torch.zeros((LAYERS, 3), dtype=torch.int64, device=device)
        self.scal = torch.zeros(2, **f64)   # amax, scale
        n = net
        self.dims = [(n.in1, n.hidden), (n.hidden, n.hidden), (n.hidden, n.vocab)]
        self.qX = [torch.empty(batch * i, **f64) for i, _ in self.dims]
        self.qW = [torch.empty(o * i, **f64) for i, o in self.dims]
        self.qG = torch.empty(batch * max(o for _, o in self.dims), **f64)
        self.x0 = torch.empty(batch * n.in1, **f64)
        self.h = [torch.empty(batch * n.hidden, **f64) for _ in range(2)]
        self.grads = [torch.zeros_like(t) for t in params]
        self.pinned = torch.empty(batch * max(n.hidden, n.vocab), dtype=torch.float64,
                                  pin_memory=True)

    # ------------------------------------------------------------ casts
    def _scale_for(self, l: int, t: int, f, x) -> Optional[object]:
        """Pass.scaleFor (Pass.java:249-271) on the device; None means 1.0."""
        p = self.p
        if f is None or p.scaling != Scaling.PER_TENSOR:
            return None
        amax, scale = self.scal[0:1], self.scal[1:2]
        amax_dev(x, amax)
        if p.amax_history <= 0:
            per_tensor_scale_dev(f, amax, scale)
        else:
            _call("drift_scale_for_dev", f.id, _tptr(amax), _tptr(self.history[l, t]),
                  self.hist_len, _tptr(self.history_count[l, t:t + 1]), _tptr(scale),
                  _stream_ptr())
        return scale

    def _cast(self, l: int, t: int, f, rm: Rounding, src, dst) -> None:
        d_scale = self._scale_for(l, t, f, src)
        quantize_dev(self.p, f, rm, src, dst, d_scale=d_scale, d_rng_state=self.state,
                     d_clamped=self.clamped[t:t + 1])
        if f is not None:
            self.cast[t] += src.numel()

    # ------------------------------------------------------------ linears
    def _linear_forward(self, l: int, x, w, b, out_buf) -> None:
        """Pass.linearForward (Pass.java:184-205)."""
        p = self.p
        f = p.input_format
        inp, out = self.dims[l]
        self._cast(l, T_X, f, p.input_rounding, x, self.qX[l])
        self._cast(l, T_W, f, p.input_rounding, w, self.qW[l])
        gemm_dev(p, self.qX[l], self.qW[l], out_buf, M=self.batch, N=out, K=inp, a_rs=inp,
                 b_rs=inp, bias=b, d_rng_state=self.state)

    def _linear_backward(self, l: int, dy, dx_buf, dw, db) -> None:
        """Pass.linearBackward (Pass.java:207-241)."""
        p = self.p
        inp, out = self.dims[l]
        B = self.batch
        qg = self.qG[:B * out]
        self._cast(l, T_G, p.grad_cast_format(), p.grad_cast_rounding(), dy, qg)
        if dx_buf is not None:
            gemm_dev(p, qg, self.qW[l], dx_buf, M=B, N=inp, K=out, a_rs=out, a_ks=1, b_rs=1,
                     b_ks=inp, d_rng_state=self.state)
        gemm_dev(p, qg, self.qX[l], dw, M=out, N=inp, K=B, a_rs=1, a_ks=out, b_rs=1, b_ks=inp,
                 d_rng_state=self.state)
        _call("drift_bias_grad_dev", _tptr(dy), B, out, _tptr(db), _stream_ptr())

    # ------------------------------------------------------------ host functions
    def _host_tanh(self, buf) -> None:
        """Math.tanh in place (Pass.java:273-277), through pinned host memory."""
        n = buf.numel()
        host = self.pinned[:n]
        host.copy_(buf)
        self.torch.cuda.current_stream().synchronize()
        h = host.numpy()
        h[:] = np.tanh(h)
        buf.copy_(host, non_blocking=True)

    # ------------------------------------------------------------ the pass
    def loss_and_grads(self, d_contexts, targets: np.ndarray) -> float:
        """Pass.lossAndGrads (Pass.java:108-113): the loss; the gradients are
        left in self.grads (device, Net.tensors order)."""
        torch = self.torch
        n, B = self.net, self.batch
        embed, w1, b1, w2, b2, w3, b3 = self.params
        st = _stream_ptr()
        _call("drift_embed_gather_dev", _tptr(d_contexts), B * n.ctx, _tptr(embed), n.vocab,
              n.emb, _tptr(self.x0), st)
        self._linear_forward(0, self.x0, w1, b1, self.h[0])
        self._host_tanh(self.h[0])
        self._linear_forward(1, self.h[0], w2, b2, self.h[1])
        self._host_tanh(self.h[1])
        logits = torch.empty(B * n.vocab, dtype=torch.float64, device=self.dev)
        self._linear_forward(2, self.h[1], w3, b3, logits)
        host = self.pinned[:B * n.vocab]
        host.copy_(logits)
        torch.cuda.current_stream().synchronize()
        loss, d_logits = softmax_xent(host.numpy().reshape(B, n.vocab).copy(), targets)

        g = self.grads
        for x in g:
            x.zero_()
        dl = torch.from_numpy(d_logits).to(self.dev)
        dh2 = torch.empty(B * n.hidden, dtype=torch.float64, device=self.dev)
        dh1 = torch.empty_like(dh2)
        dx0 = torch.empty(B * n.in1, dtype=torch.float64, device=self.dev)
        self._linear_backward(2, dl, dh2, g[5], g[6])
        _call("drift_tanh_backward_dev", _tptr(self.h[1]), _tptr(dh2), dh2.numel(), st)
        self._linear_backward(1, dh2, dh1, g[3], g[4])
        _call("drift_tanh_backward_dev", _tptr(self.h[0]), _tptr(dh1), dh1.numel(), st)
        self._linear_backward(0, dh1, dx0, g[1], g[2])
        _call("drift_embed_grad_dev", _tptr(d_contexts), B * n.ctx, _tptr(dx0), n.emb, _tptr(g[0]),
              n.vocab, st)
        return loss

    def check(self) -> None:
        """Raises for an error a kernel flagged (NaN cast into a finite
        format, a token outside the table)."""
        _lib.check(_lib.load().drift_check_dev(_lib.Context.current().handle, _stream_ptr()))


def _signed(x: int) -> int:
    x &= 0xFFFFFFFFFFFFFFFF
    return x - (1 << 64) if x >> 63 else x


class DeviceTrainer:
    """Trainer.run's step (Trainer.java:78-205) with the state on GPU
    `device`: the same token stream, Rng seeds, measurement schedule and
    records as drift_b200.mlp.train."""

    def __init__(self, policy: NumericPolicy, seed: int, *, vocab=96, ctx=32, emb=64, hidden=2048,
                 batch=64, measure_every=25, lr=1e-3, device: int = 0):
        import torch

        self.torch = torch
        self.policy = policy
        self.dev = torch.device("cuda", device)
        _lib.Context.use_device(device)
        self.vocab, self.ctx, self.batch = vocab, ctx, batch
        self.measure_every, self.lr = measure_every, float(lr)
        net = Net(vocab, ctx, emb, hidden, 1000 + seed)
        if policy.master_fp32:
            net.round_to_fp32()
        self.net = net
        self.params = [torch.from_numpy(t.copy()).to(self.dev) for t in net.tensors()]
        self.m = [torch.zeros_like(t) for t in self.params]
        self.v = [torch.zeros_like(t) for t in self.params]
        self.pas = DevicePass(policy, net, self.params, batch, 0xC0FFEE * (seed + 1), self.dev)
        self.exact = DevicePass(NumericPolicy.exact(), net, self.params, batch, 1, self.dev)
        self.tokens = np.random.default_rng(seed)
        self.step_no = 0
        self.records: List[StepRecord] = []

    def macs_per_step(self) -> int:
        """Emulated MACs of one policy pass: forward, dgrad and wgrad of the
        three linears (the exact recompute at measurement steps excluded)."""
        n = self.net
        fwd = self.batch * (n.in1 * n.hidden + n.hidden * n.hidden + n.hidden * n.vocab)
        return 3 * fwd

    def step(self) -> StepRecord:
        torch = self.torch
        self.step_no += 1
        step = self.step_no
        contexts = self.tokens.integers(0, self.vocab, size=self.batch * self.ctx)
        targets = self.tokens.integers(0, self.vocab, size=self.batch)
        d_ctx = torch.from_numpy(contexts.astype(np.int32)).to(self.dev)
        pas = self.pas
        rec = StepRecord(step, pas.loss_and_grads(d_ctx, targets))
        if step % self.measure_every == 0 or step == 1:
            rec.loss_exact = self.exact.loss_and_grads(d_ctx, targets)
            rec.cos, rec.gain, rec.rel = compare([g.cpu().numpy() for g in pas.grads],
                                                 [g.cpu().numpy() for g in self.exact.grads])
            cl = pas.clamped.cpu().numpy()
            c = pas.cast
            rec.clamp_x = cl[T_X] / c[T_X] if c[T_X] else 0.0
            rec.clamp_w = cl[T_W] / c[T_W] if c[T_W] else 0.0
            rec.clamp_g = cl[T_G] / c[T_G] if c[T_G] else 0.0
        self.records.append(rec)
        st = _stream_ptr()
        for p_, g_, m_, v_ in zip(self.params, pas.grads, self.m, self.v):
            _call("drift_adam_dev", _tptr(p_), _tptr(g_), _tptr(m_), _tptr(v_), p_.numel(), step,
                  self.lr, int(self.policy.master_fp32), st)
        return rec

    def result(self) -> Dict:
        self.pas.check()
        self.torch.cuda.synchronize()
        state = int(self.pas.state.item()) & 0xFFFFFFFFFFFFFFFF
        return {"records": self.records, "rng_state": state,
                "grads": [g.cpu().numpy() for g in self.pas.grads],
                "params": [p_.cpu().numpy() for p_ in self.params]}


def train(policy: NumericPolicy, seed: int, *, steps=25, **kw) -> Dict:
    """drift_b200.mlp.train with the state on the GPU (keyword `device`)."""
    t = DeviceTrainer(policy, seed, **kw)
    for _ in range(steps):
        t.step()
    return t.result()
