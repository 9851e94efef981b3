"""The emulated training step of the reference's MLP language model.

Host mirror of Pass (java/src/main/java/io/drift/train/Pass.java) and of the
parts of Trainer (java/src/main/java/io/drift/train/Trainer.java) the
training-step configuration drives. Every cast (Quant.quantize) and every
forward, dgrad and wgrad contraction (the Dot.dot loops of Pass.java:200-232)
runs in the CUDA engine; the embedding lookup, biases, tanh, softmax and
cross-entropy stay in double on the host, as the reference keeps them
(Pass.java:19-21), and so does the delayed-scaling amax history (3 doubles
per layer per step, Pass.java:249-271).

The arithmetic backend is pluggable so that the same pass can be run on the
engine and on a CPU restatement with identical host code; the engine's backend is the
default and the only one in this package.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np

from .fmt import MiniFloat, Rng, Rounding
from .kernel import NumericPolicy, Quant, Scaling, gemm

LAYERS = 3
T_X, T_W, T_G = 0, 1, 2


class EngineBackend:
    """Casts and contractions through the engine's host entry points."""

    name = "engine"

    def amax(self, x: np.ndarray) -> float:
        return Quant.amax(x)

    def per_tensor_scale(self, f: MiniFloat, amax: float) -> float:
        return Quant.per_tensor_scale(f, amax)

    def quantize(self, src: np.ndarray, f: Optional[MiniFloat], p: NumericPolicy, rm: Rounding,
                 scale: float, rng: Rng):
        dst = np.empty_like(src)
        clamped = Quant.quantize(src, 0, dst, 0, src.size, f, p, scale, rng, rm)
        return dst, clamped

    def gemm(self, p: NumericPolicy, M, N, K, A, a_off, a_rs, a_ks, B, b_off, b_rs, b_ks,
             bias=None, rng: Optional[Rng] = None) -> np.ndarray:
        return gemm(p, M, N, K, A, a_off, a_rs, a_ks, B, b_off, b_rs, b_ks, bias=bias, rng=rng)


@dataclass
class Net:
    """MLP parameters (java/.../train/Net.java:32-52): embedding, three linears.
    Weights are N(0, 1/fan_in) as in Net.java:48-51, drawn from a seeded
    numpy generator (the inputs are synthetic)."""

    vocab: int
    ctx: int
    emb: int
    hidden: int
    seed: int
    embed: np.ndarray = field(init=False)
    w1: np.ndarray = field(init=False)
    b1: np.ndarray = field(init=False)
    w2: np.ndarray = field(init=False)
    b2: np.ndarray = field(init=False)
    w3: np.ndarray = field(init=False)
    b3: np.ndarray = field(init=False)

    def __post_init__(self):
        self.in1 = self.ctx * self.emb
        r = np.random.default_rng(self.seed)
        self.embed = r.standard_normal(self.vocab * self.emb)
        self.w1 = r.standard_normal(self.hidden * self.in1) * (1.0 / np.sqrt(self.in1))
        self.b1 = np.zeros(self.hidden)
        self.w2 = r.standard_normal(self.hidden * self.hidden) * (1.0 / np.sqrt(self.hidden))
        self.b2 = np.zeros(self.hidden)
        self.w3 = r.standard_normal(self.vocab * self.hidden) * (1.0 / np.sqrt(self.hidden))
        self.b3 = np.zeros(self.vocab)

    def tensors(self) -> List[np.ndarray]:
        """Net.tensors order (Net.java:55-57)."""
        return [self.embed, self.w1, self.b1, self.w2, self.b2, self.w3, self.b3]

    def round_to_fp32(self) -> None:
        for t in self.tensors():
            t[:] = t.astype(np.float32)


class Pass:
    """One forward and backward pass under a policy, with its own workspace
    and amax history (Pass.java:26-90)."""

    def __init__(self, p: NumericPolicy, net: Net, batch: int, rng_seed: int, backend=None):
        self.p = p
        self.net = net
        self.batch = batch
        self.rng = Rng(rng_seed)
        self.backend = backend or EngineBackend()
        hl = max(1, p.amax_history)
        self.history = np.zeros((LAYERS, 3, hl))
        self.history_count = np.zeros((LAYERS, 3), dtype=np.int64)
        self.qX: List[Optional[np.ndarray]] = [None] * LAYERS
        self.qW: List[Optional[np.ndarray]] = [None] * LAYERS
        self.clamped = np.zeros(3, dtype=np.int64)   # X, W, G
        self.cast = np.zeros(3, dtype=np.int64)

    # ------------------------------------------------------------ forward
    def forward(self, contexts: np.ndarray, targets: np.ndarray) -> float:
        """Pass.forward (Pass.java:117-154)."""
        n = self.net
        B = self.batch
        self.x0 = n.embed.reshape(n.vocab, n.emb)[contexts.reshape(B, n.ctx)].reshape(B * n.in1)
        self.h1 = self._linear_forward(0, self.x0, n.in1, n.w1, n.b1, n.hidden)
        self.h1 = np.tanh(self.h1)
        self.h2 = self._linear_forward(1, self.h1, n.hidden, n.w2, n.b2, n.hidden)
        self.h2 = np.tanh(self.h2)
        logits = self._linear_forward(2, self.h2, n.hidden, n.w3, n.b3, n.vocab).reshape(B, n.vocab)
        loss, self.d_logits = softmax_xent(logits, targets)
        return loss

    def loss_and_grads(self, contexts: np.ndarray, targets: np.ndarray) -> tuple:
        """Pass.lossAndGrads (Pass.java:108-113): loss and the gradients in
        Net.tensors order."""
        loss = self.forward(contexts, targets)
        return loss, self._backward(contexts)

    def _backward(self, contexts: np.ndarray) -> List[np.ndarray]:
        """Pass.backward (Pass.java:156-180)."""
        n = self.net
        B = self.batch
        dh2, dw3, db3 = self._linear_backward(2, self.d_logits, n.hidden, n.vocab)
        dh2 *= 1.0 - self.h2 * self.h2
        dh1, dw2, db2 = self._linear_backward(1, dh2, n.hidden, n.hidden)
        dh1 *= 1.0 - self.h1 * self.h1
        dx0, dw1, db1 = self._linear_backward(0, dh1, n.in1, n.hidden)
        g_embed = np.zeros(n.vocab * n.emb)
        toks = contexts.reshape(B * n.ctx)
        np.add.at(g_embed.reshape(n.vocab, n.emb), toks, dx0.reshape(B * n.ctx, n.emb))
        return [g_embed, dw1, db1, dw2, db2, dw3, db3]

    # ------------------------------------------------------------ linears
    def _linear_forward(self, l, x, inp, w, b, out) -> np.ndarray:
        """Pass.linearForward (Pass.java:184-205): cast X then W on the shared
        Rng, then y[i, o] = dot(qX row i, qW row o, in) + b[o]."""
        p = self.p
        f = p.input_format
        nx, nw = self.batch * inp, out * inp
        sx = self._scale_for(l, T_X, f, x)
        sw = self._scale_for(l, T_W, f, w)
        be = self.backend
        self.qX[l], cx = be.quantize(x, f, p, p.input_rounding, sx, self.rng)
        self.qW[l], cw = be.quantize(w, f, p, p.input_rounding, sw, self.rng)
        self.clamped[T_X] += cx
        self.clamped[T_W] += cw
        if f is not None:
            self.cast[T_X] += nx
            self.cast[T_W] += nw
        y = be.gemm(p, self.batch, out, inp, self.qX[l], 0, inp, 1, self.qW[l], 0, inp, 1,
                    bias=b, rng=self.rng)
        return y.reshape(-1)

    def _linear_backward(self, l, dy, inp, out):
        """Pass.linearBackward (Pass.java:207-241): cast G, then
        dX = dY W (row i of G against column k of W) and dW = dY^T X (column o
        of G against column k of X, over the batch); bias gradients from the
        uncast dy."""
        p = self.p
        f = p.grad_cast_format()
        ng = self.batch * out
        sg = self._scale_for(l, T_G, f, dy)
        be = self.backend
        qg, cg = be.quantize(dy, f, p, p.grad_cast_rounding(), sg, self.rng)
        self.clamped[T_G] += cg
        if f is not None:
            self.cast[T_G] += ng
        B = self.batch
        dx = be.gemm(p, B, inp, out, qg, 0, out, 1, self.qW[l], 0, 1, inp, rng=self.rng)
        dw = be.gemm(p, out, inp, B, qg, 0, 1, out, self.qX[l], 0, 1, inp, rng=self.rng)
        # Bias gradients sum the batch sequentially in double (Pass.java:234-240).
        db = np.cumsum(dy.reshape(B, out), axis=0)[-1].copy()
        return dx.reshape(-1), dw.reshape(-1), db

    def _scale_for(self, l, t, f, x) -> float:
        """Pass.scaleFor (Pass.java:249-271): current scaling, or the largest
        amax of the previous amaxHistory steps (delayed scaling)."""
        p = self.p
        if f is None or p.scaling != Scaling.PER_TENSOR:
            return 1.0
        now = self.backend.amax(x)
        if p.amax_history <= 0:
            return self.backend.per_tensor_scale(f, now)
        hist = self.history[l, t]
        count = int(self.history_count[l, t])
        if count == 0:
            use = now
        else:
            use = 0.0
            for i in range(min(count, hist.size)):
                use = max(use, hist[i])
        hist[count % hist.size] = now
        self.history_count[l, t] = count + 1
        return self.backend.per_tensor_scale(f, use)


def softmax_xent(logits: np.ndarray, targets: np.ndarray):
    """Softmax cross-entropy in double (Pass.java:134-153): z summed over k in
    order, the loss over the batch in order. Returns the mean loss and the
    flat gradient of the logits."""
    B = logits.shape[0]
    mx = logits.max(axis=1, keepdims=True)
    z = np.cumsum(np.exp(logits - mx), axis=1)[:, -1:]
    log_z = np.log(z) + mx
    loss = 0.0
    for i in range(B):
        loss += float(log_z[i, 0] - logits[i, targets[i]])
    d = np.exp(logits - log_z) / B
    d[np.arange(B), targets] -= 1.0 / B
    return loss / B, d.reshape(-1)


def compare(got: List[np.ndarray], exact: List[np.ndarray]):
    """Trainer.compare (Trainer.java:272-288): cos, gain and rel over all
    tensors concatenated, each sum taken in order as the Java loop does."""
    a = np.concatenate([np.asarray(x, dtype=np.float64).reshape(-1) for x in got])
    b = np.concatenate([np.asarray(x, dtype=np.float64).reshape(-1) for x in exact])

    def total(x):
        return float(np.cumsum(x)[-1]) if x.size else 0.0

    dot, gg, ee = total(a * b), total(a * a), total(b * b)
    dd = total((a - b) * (a - b))
    return dot / np.sqrt(gg * ee), dot / ee, np.sqrt(dd / ee)


B1, B2, EPS = 0.9, 0.999, 1e-8


def adam(params, grads, m, v, step: int, lr: float, fp32: bool) -> None:
    """Trainer.adam (Trainer.java:246-269); FP32 masters round weights and
    moments to float after every update."""
    c1 = 1 - B1 ** step
    c2 = 1 - B2 ** step
    for p, g, mt, vt in zip(params, grads, m, v):
        mi = B1 * mt + (1 - B1) * g
        vi = B2 * vt + (1 - B2) * g * g
        pi = p - lr * (mi / c1) / (np.sqrt(vi / c2) + EPS)
        if fp32:
            mi = mi.astype(np.float32).astype(np.float64)
            vi = vi.astype(np.float32).astype(np.float64)
            pi = pi.astype(np.float32).astype(np.float64)
        mt[:] = mi
        vt[:] = vi
        p[:] = pi


@dataclass
class StepRecord:
    step: int
    loss: float
    loss_exact: Optional[float] = None
    cos: Optional[float] = None
    gain: Optional[float] = None
    rel: Optional[float] = None
    clamp_x: float = 0.0
    clamp_w: float = 0.0
    clamp_g: float = 0.0


def train(policy: NumericPolicy, seed: int, *, vocab=96, ctx=32, emb=64, hidden=2048, batch=64,
          steps=25, measure_every=25, lr=1e-3, backend=None, exact_backend=None) -> Dict:
    """The training-step configuration: Trainer.run (Trainer.java:78-205)
    without corpus, eval or files. Tokens are uniform over the vocabulary from
    `seed`. The policy pass's Rng seed and the exact pass's are Trainer's
    (0xC0FFEE*(seed+1) and 1, Trainer.java:85-86); the exact FP64 recompute runs
    at step 1 and every `measure_every` steps (Trainer.java:140-175)."""
    net = Net(vocab, ctx, emb, hidden, 1000 + seed)
    if policy.master_fp32:
        net.round_to_fp32()
    pas = Pass(policy, net, batch, 0xC0FFEE * (seed + 1), backend)
    exact = Pass(NumericPolicy.exact(), net, batch, 1, exact_backend or backend)
    params = net.tensors()
    m = [np.zeros_like(t) for t in params]
    v = [np.zeros_like(t) for t in params]
    tokens = np.random.default_rng(seed)
    records: List[StepRecord] = []
    grads = None
    for step in range(1, steps + 1):
        contexts = tokens.integers(0, vocab, size=batch * ctx)
        targets = tokens.integers(0, vocab, size=batch)
        loss, grads = pas.loss_and_grads(contexts, targets)
        rec = StepRecord(step, loss)
        if step % measure_every == 0 or step == 1:
            loss_e, g_e = exact.loss_and_grads(contexts, targets)
            rec.loss_exact = loss_e
            rec.cos, rec.gain, rec.rel = compare(grads, g_e)
            c = pas.cast
            rec.clamp_x = pas.clamped[T_X] / c[T_X] if c[T_X] else 0.0
            rec.clamp_w = pas.clamped[T_W] / c[T_W] if c[T_W] else 0.0
            rec.clamp_g = pas.clamped[T_G] / c[T_G] if c[T_G] else 0.0
        records.append(rec)
        adam(params, grads, m, v, step, lr, policy.master_fp32)
    return {"records": records, "rng_state": pas.rng.state(), "grads": grads, "net": net}
