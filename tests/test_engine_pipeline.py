"""The host-buffer entry points above their pipelining thresholds
(drift_gemm from 1024 rows, with B in column blocks from 1024 columns;
drift_quantize from 4M elements): operands cross in chunks whose copies
overlap the kernels, and the results stay bit-exact
against the oracle, ragged last chunks, offsets, strides and bias included."""
import numpy as np
import pytest

from helpers import assert_bits, heavy_tailed, opolicy
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def d():
    import drift_b200
    return drift_b200


@pytest.mark.parametrize("acc,order", [(0, 0), (1, 0), (2, 2), (3, 3), (1, 1)])
def test_gemm_row_chunks(d, acc, order):
    rs = np.random.default_rng(acc * 5 + order)
    M, N, K, a_rs, a_off = 1100, 70, 33, 41, 5      # ragged last chunk, padded rows
    A = heavy_tailed(rs, a_off + M * a_rs)
    B = heavy_tailed(rs, N * K)
    bias = heavy_tailed(rs, N)
    p = d.NumericPolicy.builder("t").acc(d.Acc(acc)).order(d.Order(order)).build()
    out = np.full((M, N + 3), 9.0)[:, :N]           # strided C rows
    got = d.gemm(p, M, N, K, A, a_off, a_rs, 1, B, 0, K, 1, bias=bias, out=out)
    want, _ = O.gemm(opolicy(p), M, N, K, A, a_off, a_rs, 1, B, 0, K, 1, bias=bias, threads=16)
    assert_bits(got, want)


@pytest.mark.parametrize("acc,order", [(0, 0), (1, 0), (2, 2), (3, 3), (2, 1)])
def test_gemm_row_chunks_and_b_blocks(d, acc, order):
    """Both operands row-major and 1024+ long: B crosses in four column blocks
    (320, 320, 320, 140 rows of B) behind A's first row chunk, which is
    contracted block by block; then a column-strided B, which crosses whole."""
    rs = np.random.default_rng(acc * 7 + order + 1)
    M, N, K, a_rs, a_off, b_rs, b_off = 1100, 1100, 33, 41, 5, 37, 3
    A = heavy_tailed(rs, a_off + M * a_rs)
    B = heavy_tailed(rs, b_off + N * b_rs)
    bias = heavy_tailed(rs, N)
    p = d.NumericPolicy.builder("t").acc(d.Acc(acc)).order(d.Order(order)).build()
    out = np.full((M, N + 3), 9.0)[:, :N]           # strided C rows
    got = d.gemm(p, M, N, K, A, a_off, a_rs, 1, B, b_off, b_rs, 1, bias=bias, out=out)
    want, _ = O.gemm(opolicy(p), M, N, K, A, a_off, a_rs, 1, B, b_off, b_rs, 1, bias=bias,
                     threads=16)
    assert_bits(got, want, "B in column blocks")
    Bt = heavy_tailed(rs, K * N)                     # B read down its columns
    got = d.gemm(p, M, N, K, A, a_off, a_rs, 1, Bt, 0, 1, N, bias=bias)
    want, _ = O.gemm(opolicy(p), M, N, K, A, a_off, a_rs, 1, Bt, 0, 1, N, bias=bias, threads=16)
    assert_bits(got, want, "B whole")


@pytest.mark.parametrize("name", ["fp8", "fp8-mx", "mxfp4", "bf16"])
def test_quantize_chunks(d, name):
    rs = np.random.default_rng(len(name))
    n = (1 << 22) + 12345
    src = heavy_tailed(rs, n)
    src[::1001] = 0.0
    p = d.policies.by_name(name)
    f = p.input_format
    scale = d.Quant.per_tensor_scale(f, d.Quant.amax(src)) if p.scaling == d.Scaling.PER_TENSOR \
        else 1.0
    dst = np.empty(n)
    clamped = d.Quant.quantize(src, 0, dst, 0, n, f, p, scale, None)
    want, wc, _ = O.quantize(opolicy(p), f.id, int(p.input_rounding), src, scale, None)
    assert_bits(dst, want)
    assert clamped == wc


def test_quantize_mx_odd_block(d):
    """An MX block length that does not divide the chunk unit's power of two."""
    rs = np.random.default_rng(9)
    n = (1 << 22) + 999
    src = heavy_tailed(rs, n)
    p = d.policies.by_name("fp8-mx").to_builder("mx37").scale_block(37).build()
    dst = np.empty(n)
    clamped = d.Quant.quantize(src, 0, dst, 0, n, p.input_format, p, 1.0, None)
    want, wc, _ = O.quantize(opolicy(p), p.input_format.id, 0, src, 1.0, None)
    assert_bits(dst, want)
    assert clamped == wc
