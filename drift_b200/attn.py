"""The emulated training step of the reference's attention model.

Host mirror of AttnNet and AttnPass (java/src/main/java/io/drift/train/AttnNet.java,
AttnPass.java): one block of causal single-head self attention and an MLP with
residual connections. Every cast (Quant.quantize) and every matmul runs in the
CUDA engine: the seven linears as drift_gemm, and the four attention matmuls
(scores, context, and their gradients, the Dot.dot loops of AttnPass.java:245-290
and :373-427) as drift_contract with causal masks and ragged per-row windows.
The embedding lookup, residual adds, softmax, ReLU and loss stay in double on
the host, as the reference keeps them (AttnPass.java:21-24), and so do the
per-cast statistics of countUnderflow (:555-613).

A stochastic accumulator shares the pass's Rng with the casts, so the calls run
in the reference's order: in the backward pass the dProb and dv loops (and the
dq and dk loops) alternate per batch element (:373-389, :410-425).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

from .fmt import MiniFloat, Rng, Rounding
from .kernel import (Acc, NumericPolicy, Rounding as _R, Scaling, Window, contract, contraction)
from .mlp import EngineBackend as _MlpBackend


class EngineBackend(_MlpBackend):
    """Casts, linears and attention contractions through the engine."""

    def contract(self, p: NumericPolicy, op, A, B, C, rng: Optional[Rng] = None):
        return contract(p, op, A, B, C, rng=rng)


TENSOR_NAMES = ("embed", "pos", "wq", "wk", "wv", "wo", "w1", "b1", "w2", "b2", "wout", "bout")


@dataclass
class AttnNet:
    """AttnNet parameters (AttnNet.java:42-74): N(0, 1/sqrt(dim)) embeddings
    and d-input weights, N(0, 0.02) positions, N(0, 1/sqrt(hidden)) for w2,
    zero biases; drawn from a seeded numpy generator (synthetic inputs)."""

    vocab: int
    ctx: int
    dim: int
    hidden: int
    seed: int
    tensors_: List[np.ndarray] = field(init=False, repr=False)

    def __post_init__(self):
        r = np.random.default_rng(self.seed)
        v, t, d, h = self.vocab, self.ctx, self.dim, self.hidden
        s = 1.0 / math.sqrt(d)
        self.embed = r.standard_normal(v * d) * s
        self.pos = r.standard_normal(t * d) * 0.02
        self.wq = r.standard_normal(d * d) * s
        self.wk = r.standard_normal(d * d) * s
        self.wv = r.standard_normal(d * d) * s
        self.wo = r.standard_normal(d * d) * s
        self.w1 = r.standard_normal(h * d) * s
        self.b1 = np.zeros(h)
        self.w2 = r.standard_normal(d * h) * (1.0 / math.sqrt(h))
        self.b2 = np.zeros(d)
        self.wout = r.standard_normal(v * d) * s
        self.bout = np.zeros(v)

    def tensors(self) -> List[np.ndarray]:
        """AttnNet.tensors order (AttnNet.java:76-79)."""
        return [getattr(self, n) for n in TENSOR_NAMES]

    def round_to_fp32(self) -> None:
        for x in self.tensors():
            x[:] = x.astype(np.float32)


class AttnPass:
    """One forward and backward pass under a policy (AttnPass.java:26-197).
    Scaling is always current (the reference does not wire delayed scaling
    into this model, :20-23)."""

    def __init__(self, p: NumericPolicy, net: AttnNet, batch: int, rng_seed: int, backend=None):
        self.p = p
        self.net = net
        self.batch = batch
        self.rng = Rng(rng_seed)
        self.backend = backend or EngineBackend()
        self.t, self.d, self.h, self.v = net.ctx, net.dim, net.hidden, net.vocab
        self.rows = batch * self.t
        self.score_scale = 1.0 / math.sqrt(self.d)
        self.sr_acc = p.acc_rounding == _R.STOCHASTIC and p.acc in (Acc.FP16, Acc.BF16)
        wide = self.rows * max(self.d, self.h, self.v)
        self.qg_rows = np.zeros(wide)
        self.qg_wide = np.zeros(wide)
        for name in ("clamped_x", "clamped_w", "clamped_g", "cast_x", "cast_w", "cast_g",
                     "clamped_prob", "cast_prob", "underflowed", "spread_count", "cast_err_count",
                     "block_spread_count", "cast_bias_count"):
            setattr(self, name, 0)
        self.spread_sum = self.cast_err_sum = self.block_spread_sum = self.cast_bias_sum = 0.0

    # ------------------------------------------------------------ counters
    def clamp_counts(self) -> List[int]:
        """AttnPass.clampCounts (:186-194), doubles as their raw bits."""
        def bits(x):
            return int(np.float64(x).view(np.int64))
        mean = lambda s, c: s / c if c else 0.0
        return [self.clamped_x, self.cast_x, self.clamped_w, self.cast_w, self.clamped_g,
                self.cast_g, self.clamped_prob, self.cast_prob, self.underflowed,
                self.cast_x + self.cast_w + self.cast_g,
                int(mean(self.spread_sum, self.spread_count)), self.spread_count,
                bits(mean(self.cast_err_sum, self.cast_err_count)),
                bits(mean(self.block_spread_sum, self.block_spread_count)),
                bits(mean(self.cast_bias_sum, self.cast_bias_count))]

    # ------------------------------------------------------------ forward
    def loss_and_grads(self, contexts: np.ndarray, targets: np.ndarray):
        loss = self.forward(contexts, targets)
        return loss, self._backward(contexts)

    def forward(self, contexts: np.ndarray, targets: np.ndarray) -> float:
        """AttnPass.forward (:210-332)."""
        n, p = self.net, self.p
        B, t, d, h, v, rows = self.batch, self.t, self.d, self.h, self.v, self.rows
        tok = np.asarray(contexts).reshape(B, t)
        self.x = (n.embed.reshape(v, d)[tok] + n.pos.reshape(t, d)[None]).reshape(-1)

        self.qx = self._cast_act(self.x)
        self.qWq = self._cast_weight(n.wq)
        self.qWk = self._cast_weight(n.wk)
        self.qWv = self._cast_weight(n.wv)
        q = self._linear(self.qx, self.qWq, None, rows, d, d)
        k = self._linear(self.qx, self.qWk, None, rows, d, d)
        val = self._linear(self.qx, self.qWv, None, rows, d, d)

        if p.cast_scores:
            self.qq = self._cast_act(q)
            self.qk = self._cast_act(k)
        else:
            self.qq, self.qk = q.copy(), k.copy()
        scores = np.zeros(B * t * t)
        self.backend.contract(p, contraction(
            batch=B, rows=t, cols=t, depth=d, a_batch=t * d, a_row=d, a_k=1, b_batch=t * d,
            b_col=d, b_k=1, c_batch=t * t, c_row=t, alpha=self.score_scale, causal=True),
            self.qq, self.qk, scores, self.rng)
        self.prob = _causal_softmax(scores.reshape(B, t, t)).reshape(-1)

        if p.cast_probs:
            self.qprob = self._cast_probabilities(self.prob)
            self.qv = self._cast_act(val)
        else:
            self.qprob, self.qv = self.prob.copy(), val.copy()
        ctxv = np.zeros(rows * d)
        self.backend.contract(p, contraction(
            batch=B, rows=t, cols=d, depth=t, a_batch=t * t, a_row=t, a_k=1, b_batch=t * d,
            b_col=1, b_k=d, c_batch=t * d, c_row=d, window=Window.PREFIX),
            self.qprob, self.qv, ctxv, self.rng)

        self.qctxv = self._cast_act(ctxv)
        self.qWo = self._cast_weight(n.wo)
        attn_out = self._linear(self.qctxv, self.qWo, None, rows, d, d)
        self.hres = self.x + attn_out

        self.qh = self._cast_act(self.hres)
        self.qW1 = self._cast_weight(n.w1)
        self.z1 = self._linear(self.qh, self.qW1, n.b1, rows, d, h)
        # Math.max(0.0, z): NaN stays NaN, -0.0 becomes 0.0.
        m1 = np.where(np.isnan(self.z1), self.z1, np.where(self.z1 > 0.0, self.z1, 0.0))
        self.qm1 = self._cast_act(m1)
        self.qW2 = self._cast_weight(n.w2)
        y = self._linear(self.qm1, self.qW2, n.b2, rows, h, d) + self.hres

        self.qy = self._cast_act(y)
        self.qWout = self._cast_weight(n.wout)
        logits = self._linear(self.qy, self.qWout, n.bout, rows, d, v).reshape(rows, v)

        mx = logits.max(axis=1, keepdims=True)
        z = np.cumsum(np.exp(logits - mx), axis=1)[:, -1:]
        log_z = np.log(z) + mx
        tg = np.asarray(targets).reshape(rows)
        loss = 0.0
        for r in range(rows):
            loss += float(log_z[r, 0] - logits[r, tg[r]])
        dl = np.exp(logits - log_z) / rows
        dl[np.arange(rows), tg] -= 1.0 / rows
        self.d_logits = dl.reshape(-1)
        return loss / rows

    # ------------------------------------------------------------ backward
    def _backward(self, contexts: np.ndarray) -> List[np.ndarray]:
        """AttnPass.backward (:334-438): gradients in AttnNet.tensors order."""
        n, p = self.net, self.p
        B, t, d, h, v, rows = self.batch, self.t, self.d, self.h, self.v, self.rows
        g = [np.zeros_like(x) for x in n.tensors()]

        qg = self._cast_grad(self.d_logits, self.qg_wide)
        dy = self._dinput(qg, self.qWout, rows, d, v)
        g[10] = self._dweight(qg, self.qy, rows, d, v)
        g[11] = _dbias(self.d_logits, rows, v)

        dh = dy.copy()
        qg = self._cast_grad(dy, self.qg_rows)
        dm1 = self._dinput(qg, self.qW2, rows, h, d)
        g[8] = self._dweight(qg, self.qm1, rows, h, d)
        g[9] = _dbias(dy, rows, d)

        dz1 = np.where(self.z1 > 0.0, dm1, 0.0)
        qg = self._cast_grad(dz1, self.qg_wide)
        dh = dh + self._dinput(qg, self.qW1, rows, d, h)
        g[6] = self._dweight(qg, self.qh, rows, d, h)
        g[7] = _dbias(dz1, rows, h)

        dx = dh.copy()
        qg = self._cast_grad(dh, self.qg_rows)
        d_ctxv = self._dinput(qg, self.qWo, rows, d, d)
        g[5] = self._dweight(qg, self.qctxv, rows, d, d)

        if p.cast_probs:
            qgw = self._cast_grad(d_ctxv, self.qg_wide)
        else:
            self.qg_wide[:rows * d] = d_ctxv
            qgw = self.qg_wide
        d_prob = np.zeros(B * t * t)
        dv = np.zeros(rows * d)
        dprob_op = dict(rows=t, cols=t, depth=d, a_batch=t * d, a_row=d, a_k=1, b_batch=t * d,
                        b_col=d, b_k=1, c_batch=t * t, c_row=t, causal=True)
        dv_op = dict(rows=t, cols=d, depth=t, a_batch=t * t, a_row=1, a_k=t, b_batch=t * d,
                     b_col=1, b_k=d, c_batch=t * d, c_row=d, window=Window.SUFFIX)
        self._pair_loops(dprob_op, qgw, self.qv, d_prob, dv_op, self.qprob, qgw, dv)

        d_score = _softmax_backward(self.prob.reshape(B, t, t), d_prob.reshape(B, t, t),
                                    self.score_scale).reshape(-1)
        qgs = self._cast_grad(d_score, np.zeros(B * t * t)) if p.cast_scores else d_score
        dq = np.zeros(rows * d)
        dk = np.zeros(rows * d)
        dq_op = dict(rows=t, cols=d, depth=t, a_batch=t * t, a_row=t, a_k=1, b_batch=t * d,
                     b_col=1, b_k=d, c_batch=t * d, c_row=d, window=Window.PREFIX)
        dk_op = dict(rows=t, cols=d, depth=t, a_batch=t * t, a_row=1, a_k=t, b_batch=t * d,
                     b_col=1, b_k=d, c_batch=t * d, c_row=d, window=Window.SUFFIX)
        self._pair_loops(dq_op, qgs, self.qk, dq, dk_op, qgs, self.qq, dk)

        for grad_out, qw, slot in ((dq, self.qWq, 2), (dk, self.qWk, 3), (dv, self.qWv, 4)):
            qg = self._cast_grad(grad_out, self.qg_rows)       # projBackward (:441-445)
            dx = dx + self._dinput(qg, qw, rows, d, d)
            g[slot] = self._dweight(qg, self.qx, rows, d, d)

        tok = np.asarray(contexts).reshape(rows)
        dxr = dx.reshape(rows, d)
        np.add.at(g[0].reshape(v, d), tok, dxr)
        np.add.at(g[1].reshape(t, d), np.tile(np.arange(t), B), dxr)
        return g

    def _pair_loops(self, op1, a1, b1, c1, op2, a2, b2, c2) -> None:
        """Two contractions that the reference interleaves per batch element.
        Their order matters only when the accumulator draws."""
        be, p = self.backend, self.p
        if not self.sr_acc:
            be.contract(p, contraction(batch=self.batch, **op1), a1, b1, c1, self.rng)
            be.contract(p, contraction(batch=self.batch, **op2), a2, b2, c2, self.rng)
            return
        for b in range(self.batch):
            for op, a, bb, c in ((op1, a1, b1, c1), (op2, a2, b2, c2)):
                one = dict(op, a_off=b * op["a_batch"], b_off=b * op["b_batch"],
                           c_off=b * op["c_batch"])
                be.contract(p, contraction(**one), a, bb, c, self.rng)

    # ------------------------------------------------------------ matmuls
    def _linear(self, qin, qw, bias, r, inp, out) -> np.ndarray:
        """AttnPass.linear (:449-456): dot + bias[o], or + 0.0 without a bias."""
        b = bias if bias is not None else np.zeros(out)
        return self.backend.gemm(self.p, r, out, inp, qin, 0, inp, 1, qw, 0, inp, 1, bias=b,
                                 rng=self.rng).reshape(-1)

    def _dinput(self, qg, qw, r, inp, out) -> np.ndarray:
        """AttnPass.dInput (:459-471): row i of G against column c of W."""
        return self.backend.gemm(self.p, r, inp, out, qg, 0, out, 1, qw, 0, 1, inp,
                                 rng=self.rng).reshape(-1)

    def _dweight(self, qg, qin, r, inp, out) -> np.ndarray:
        """AttnPass.dWeight (:474-481): column o of G against column c of X."""
        return self.backend.gemm(self.p, out, inp, r, qg, 0, 1, out, qin, 0, 1, inp,
                                 rng=self.rng).reshape(-1)

    # ------------------------------------------------------------ casts
    def _cast_probabilities(self, src):
        f = self.p.input_format
        dst, clamped = self._cast(src, src.size, f, self.p.input_rounding)
        self.clamped_x += clamped
        self.clamped_prob += clamped
        if f is not None:
            self.cast_x += src.size
            self.cast_prob += src.size
        return dst

    def _cast_act(self, src):
        f = self.p.input_format
        dst, clamped = self._cast(src, src.size, f, self.p.input_rounding)
        self.clamped_x += clamped
        if f is not None:
            self.cast_x += src.size
        return dst

    def _cast_weight(self, src):
        f = self.p.input_format
        dst, clamped = self._cast(src, src.size, f, self.p.input_rounding)
        self.clamped_w += clamped
        if f is not None:
            self.cast_w += src.size
        return dst

    def _cast_grad(self, src, buf):
        """castGrad into the shared buffer `buf` (:531-537): its first n
        elements are overwritten, the rest keep what earlier casts left."""
        f = self.p.grad_cast_format()
        dst, clamped = self._cast(src, src.size, f, self.p.grad_cast_rounding())
        self.clamped_g += clamped
        if f is not None:
            self.cast_g += src.size
        buf[:src.size] = dst
        return buf

    def _cast(self, src, n, f: Optional[MiniFloat], rm: Rounding):
        """AttnPass.cast (:539-549)."""
        be, p = self.backend, self.p
        scale = 1.0
        if f is not None and p.scaling == Scaling.PER_TENSOR:
            scale = be.per_tensor_scale(f, be.amax(src))
        dst, clamped = be.quantize(src, f, p, rm, scale, self.rng)
        if f is not None:
            self._count_underflow(src, dst)
        return dst, clamped

    def _count_underflow(self, src, dst) -> None:
        """AttnPass.countUnderflow (:556-613), its sums in the Java order."""
        a = np.abs(src)
        self.underflowed += int(np.count_nonzero((src != 0.0) & (dst == 0.0)))
        mx = float(a.max()) if a.size else 0.0
        nz = a[a != 0.0]
        mn = float(nz.min()) if nz.size else np.finfo(np.float64).max
        if mx > 0.0 and mn < np.finfo(np.float64).max:
            self.spread_sum += math.log(mx / mn) / math.log(2.0)
            self.spread_count += 1
        e = dst - src
        num = _seq_sum(e * e)
        den = _seq_sum(src * src)
        proj = _seq_sum(e * src)
        if den > 0.0:
            self.cast_err_sum += math.sqrt(num / den)
            self.cast_err_count += 1
            self.cast_bias_sum += proj / den
            self.cast_bias_count += 1
        block = self.p.scale_block
        for start in range(0, src.size, block):
            blk = a[start:start + block]
            bmax = float(blk.max())
            bnz = blk[blk != 0.0]
            if bmax > 0.0 and bnz.size:
                self.block_spread_sum += math.log(bmax / float(bnz.min())) / math.log(2.0)
                self.block_spread_count += 1


def _seq_sum(x: np.ndarray) -> float:
    """A left-to-right double sum, as a Java loop adds."""
    return float(np.cumsum(x)[-1]) if x.size else 0.0


def _causal_softmax(scores: np.ndarray) -> np.ndarray:
    """The softmax of AttnPass.forward (:256-270) over s <= i, 0.0 above."""
    B, t, _ = scores.shape
    prob = np.zeros_like(scores)
    for i in range(t):
        s = scores[:, i, :i + 1]
        mx = s.max(axis=1, keepdims=True)
        e = np.exp(s - mx)
        z = np.cumsum(e, axis=1)[:, -1:]
        prob[:, i, :i + 1] = e / z
    return prob


def _softmax_backward(prob: np.ndarray, d_prob: np.ndarray, scale: float) -> np.ndarray:
    """AttnPass.java:392-407: dScore = prob * (dProb - sum) * scale on s <= i."""
    B, t, _ = prob.shape
    out = np.zeros_like(prob)
    for i in range(t):
        pr, dp = prob[:, i, :i + 1], d_prob[:, i, :i + 1]
        s = np.cumsum(pr * dp, axis=1)[:, -1:]
        out[:, i, :i + 1] = pr * (dp - s) * scale
    return out


def _dbias(d_out: np.ndarray, r: int, out: int) -> np.ndarray:
    """AttnPass.dBias (:484-493): the uncast gradient summed over rows in order."""
    return np.cumsum(d_out.reshape(r, out), axis=0)[-1].copy()
