// gemm32.cu — the FP32 accumulator over narrow products, on the FP32 pipe.
//
// Dot.forward's FP32 loop (java/src/main/java/io/drift/kernel/Dot.java:50-56)
// computes s = (float)(s + a*b): the product rounded to double, the sum
// rounded to double, then to float. When a and b are fp32 numbers whose exact
// product is an fp32 number too, the product is exact and s + a*b is a sum of
// two floats. Rounding such a sum first to 53 bits and then to 24 gives the
// same float as rounding it once to 24 bits, because 53 >= 2*24 + 2 (S. A.
// Figueroa, "When is double rounding innocuous?", ACM SIGNUM Newsletter 30(3),
// 1995). So the whole chain is fmaf(a, b, s) with every FMA exact to the
// Java result, and one FFMA does the work of a DMUL, a DADD and the rounding.
// The same holds for the reversed walk (Dot.java:72-84) and for BLOCKED's fold
// (float)(total + partial) of two floats (Dot.java:115-118).
//
// When it applies. The product of a = ma*2^la and b = mb*2^lb (odd ma, mb) is
// ma*mb*2^(la+lb), an fp32 number when ma*mb has at most 24 bits, la + lb >=
// -149 (fp32's last subnormal bit) and |a*b| < 2^128. A scan of each operand
// records its widest significand, its largest exponent and its lowest set bit
// (and whether it holds Inf or NaN); a one-thread decision combines the two
// operands' bounds, which cover every pair:
//   width(A) + width(B) <= 24, low(A) + low(B) >= -149, top(A) + top(B) <= 126,
// and each operand alone is fp32-representable. Those are the shapes of the
// bf16 and MX-scaled minifloat casts (8- and 4-bit significands on power-of-two
// scales); a per-tensor scale that is not a power of two widens the values to
// 53 bits and leaves them on the double-precision contraction.
//
// The decision stays on the device: the scan and decision are queued, then
// both contractions, and each reads the decision word first and leaves at once
// unless it is its turn. Nothing waits on the host.
//
// Layout. The scan also transposes each operand into k-major fp32 rows (row k
// holds every output row's k-th term, padded to a multiple of 4 floats), so a
// k step of a 128-row tile is 512 contiguous bytes. A CTA of 256 threads owns
// a 128 x 128 output tile and each thread an 8 x 8 block (rows ty*4 + {0..3}
// and 64 + ty*4 + {0..3}, columns likewise with tx), fed by four 16-byte
// shared-memory loads per k for 64 FMAs. K advances in tiles of 16 through a
// 4-stage ring filled by TMA (one 128 x 16 box per operand per stage, zero
// fill past the edges; a zero term adds +0, which leaves every sum unchanged
// because no chain here ever holds -0: it starts at +0 and x + (-x) is +0).
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "internal.h"
#include "tma.cuh"

namespace drift {

constexpr int F_BM = 128, F_BN = 128, F_BK = 16, F_THREADS = 256, F_STAGES = 4;
constexpr int F_TILE_FLOATS = F_BK * F_BM;                    // one operand, one stage
constexpr unsigned F_TILE_BYTES = F_TILE_FLOATS * sizeof(float);  // 8 KiB
constexpr int F_SMEM = F_STAGES * 2 * F_TILE_FLOATS * (int)sizeof(float) + 64;
// Below this many multiply-accumulates the scan costs more than it can save.
constexpr double kF32MinMacs = 134217728.0;  // 2^27
// Workspace ceiling for the two transposed operands.
constexpr size_t kF32MaxBytes = size_t(16) << 30;

// Scan results per operand, each kept as a maximum so that zero is the
// identity: [0] widest significand in bits, [1] largest exponent + kExpBias,
// [2] kExpBias - lowest set bit's exponent, [3] 1 if any Inf or NaN.
// An operand of zeros only leaves [1] == 0.
constexpr int kExpBias = 1100;
constexpr int kPropWords = 4;
constexpr int kFlagWord = 2 * kPropWords;  // the decision: 1 = this path, 0 = the other

// Folds one element into the running scan maxima.
__device__ __forceinline__ void scan_one(double x, int &wide, int &top, int &low, int &bad) {
    const uint64_t u = dbits(x) & 0x7FFFFFFFFFFFFFFFULL;
    if (u == 0) return;
    const int ef = (int)(u >> 52);
    if (ef == 0x7FF) {
        bad = 1;
        return;
    }
    uint64_t m = u & 0xFFFFFFFFFFFFFULL;
    int e, lsb;
    if (ef) {
        m |= 1ULL << 52;  // value = m * 2^(ef - 1075)
        e = ef - 1023;
        lsb = ef - 1075 + (__ffsll((long long)m) - 1);
    } else {  // subnormal: value = m * 2^-1074
        e = -1074 + (63 - __clzll((long long)m));
        lsb = -1074 + (__ffsll((long long)m) - 1);
    }
    wide = max(wide, e - lsb + 1);
    top = max(top, e + kExpBias);
    low = max(low, kExpBias - lsb);
}

// Transposes X (rows x K; element (r, k) at X[r*rs + k*ks]) into
// Xt[k*ld + r] as floats through 32 x 32 shared-memory tiles, and folds every
// element into the operand's scan words. Grid-stride over tiles; one set of
// atomics per warp.
__global__ void __launch_bounds__(256) scan_pack_kernel(const double *X, int64_t rows, int64_t K,
                                                        int64_t rs, int64_t ks, float *Xt,
                                                        int64_t ld, int *props) {
    __shared__ float tile[32][33];
    const int lane = threadIdx.x & 31, wy = threadIdx.x >> 5;
    const int64_t tr = (rows + 31) / 32, tk = (K + 31) / 32;
    const bool kfast = ks == 1 || rs != 1;  // coalesce the reads along the unit stride
    int wide = 0, top = 0, low = 0, bad = 0;
    for (int64_t t = blockIdx.x; t < tr * tk; t += gridDim.x) {
        const int64_t r0 = (t % tr) * 32, k0 = (t / tr) * 32;
#pragma unroll
        for (int q = wy; q < 32; q += 8) {
            const int i = kfast ? q : lane, j = kfast ? lane : q;  // row, k within the tile
            const int64_t r = r0 + i, k = k0 + j;
            float f = 0.0f;
            if (r < rows && k < K) {
                const double x = X[r * rs + k * ks];
                scan_one(x, wide, top, low, bad);
                f = __double2float_rn(x);  // exact whenever the decision picks this path
            }
            tile[j][i] = f;
        }
        __syncthreads();
#pragma unroll
        for (int q = wy; q < 32; q += 8) {
            const int64_t k = k0 + q, r = r0 + lane;
            if (k < K && r < rows) Xt[k * ld + r] = tile[q][lane];
        }
        __syncthreads();
    }
    wide = __reduce_max_sync(0xFFFFFFFFu, wide);
    top = __reduce_max_sync(0xFFFFFFFFu, top);
    low = __reduce_max_sync(0xFFFFFFFFu, low);
    bad = __reduce_max_sync(0xFFFFFFFFu, bad);
    if (lane == 0) {
        if (wide) atomicMax(&props[0], wide);
        if (top) atomicMax(&props[1], top);
        if (low) atomicMax(&props[2], low);
        if (bad) atomicMax(&props[3], bad);
    }
}

// Combines the two operands' scans into the decision word (and the context's
// route word, when given).
__global__ void f32_decide_kernel(int *props, int *route) {
    const int *a = props, *b = props + kPropWords;
    bool ok = !a[3] && !b[3];
    const bool za = a[1] == 0, zb = b[1] == 0;
    const int wa = a[0], wb = b[0];
    const int ta = a[1] - kExpBias, tb = b[1] - kExpBias;
    const int la = kExpBias - a[2], lb = kExpBias - b[2];
    // Each element is an fp32 number: at most 24 bits, none below 2^-149, none
    // at or above 2^128.
    if (!za) ok = ok && wa <= 24 && la >= -149 && ta <= 127;
    if (!zb) ok = ok && wb <= 24 && lb >= -149 && tb <= 127;
    // Each product is one: |a| < 2^(ta+1) and |b| < 2^(tb+1) bound it below
    // 2^(ta+tb+2), and a product of at most 24 bits below 2^128 is finite.
    if (!za && !zb) ok = ok && wa + wb <= 24 && la + lb >= -149 && ta + tb + 2 <= 128;
    props[kFlagWord] = ok ? 1 : 0;
    if (route) *route = ok ? DRIFT_ROUTE_FP32 : DRIFT_ROUTE_SCANNED;
}

struct F32Args {
    int64_t M, N, K;
    int64_t acc_block;  // BLOCKED chunk, a multiple of F_BK
    const double *bias;
    double *C;
    int64_t c_rs;
    const int *flag;
    int *err;
};

template <int ORDER>
__global__ void __launch_bounds__(F_THREADS, ORDER == DRIFT_BLOCKED ? 1 : 2)
    gemm_f32_kernel(const F32Args g, const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmB) {
    if (*g.flag != 1) return;  // the double-precision contraction has this call
    extern __shared__ __align__(128) float fsm[];
    uint64_t *bars = reinterpret_cast<uint64_t *>(fsm + F_STAGES * 2 * F_TILE_FLOATS);
    constexpr bool REV = ORDER == DRIFT_REVERSED;
    constexpr bool BLOCK = ORDER == DRIFT_BLOCKED;

    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    // M, N and K are below 2^31 (checked on the host), so 32-bit indices do.
    const int m0 = (int)blockIdx.y * F_BM;
    const int n0 = (int)blockIdx.x * F_BN;
    const int T = (int)((g.K + F_BK - 1) / F_BK);

    float acc[8][8], tot[BLOCK ? 8 : 1][BLOCK ? 8 : 1];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;
    if constexpr (BLOCK) {
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) tot[i][j] = 0.0f;
    }

    // TMA writes need 128-byte-aligned destinations; every stage offset is a
    // multiple of 8 KiB, so only the base is checked.
    if ((smem_addr(fsm) & 127u) != 0) {
        if (tid == 0) atomicOr(g.err, DEV_ERR_TIMEOUT);
        return;
    }
    if (tid == 0) {
        for (int s = 0; s < F_STAGES; s++) mbar_init(&bars[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    auto issue = [&](int it) {
        if (it < T && tid == 0) {
            const int t = REV ? T - 1 - it : it;
            const int s = it % F_STAGES;
            float *sA = fsm + s * 2 * F_TILE_FLOATS;
            mbar_expect_tx(&bars[s], 2 * F_TILE_BYTES);
            tma_load_2d(sA, &tmA, m0, t * F_BK, &bars[s]);
            tma_load_2d(sA + F_TILE_FLOATS, &tmB, n0, t * F_BK, &bars[s]);
        }
    };

    for (int s = 0; s < F_STAGES - 1; s++) issue(s);
    for (int it = 0; it < T; it++) {
        const int s = it % F_STAGES;
        // Warp 0 watches the stage; the CTA barrier then orders the landed tile
        // before every read, tells every thread the previous stage is free, and
        // makes the CTA leave together if the stage timed out.
        bool lost = false;
        if (tid < 32) lost = !mbar_wait(&bars[s], (unsigned)((it / F_STAGES) & 1));
        if (__syncthreads_or(lost)) {
            if (tid == 0) {
                atomicOr(g.err, DEV_ERR_TIMEOUT);
                for (int j = it; j < T && j < it + F_STAGES - 1; j++)
                    mbar_wait(&bars[j % F_STAGES], (unsigned)((j / F_STAGES) & 1));
            }
            return;
        }
        issue(it + F_STAGES - 1);
        const float *sA = fsm + s * 2 * F_TILE_FLOATS;
        const float *sB = sA + F_TILE_FLOATS;
#pragma unroll
        for (int q = 0; q < F_BK; q++) {
            const int kk = REV ? F_BK - 1 - q : q;
            const float4 a0 = *reinterpret_cast<const float4 *>(sA + kk * F_BM + ty * 4);
            const float4 a1 = *reinterpret_cast<const float4 *>(sA + kk * F_BM + 64 + ty * 4);
            const float4 b0 = *reinterpret_cast<const float4 *>(sB + kk * F_BN + tx * 4);
            const float4 b1 = *reinterpret_cast<const float4 *>(sB + kk * F_BN + 64 + tx * 4);
            const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
        }
        if constexpr (BLOCK) {
            if (((int64_t)(it + 1) * F_BK) % g.acc_block == 0) {
#pragma unroll
                for (int i = 0; i < 8; i++)
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        tot[i][j] = __fadd_rn(tot[i][j], acc[i][j]);
                        acc[i][j] = 0.0f;
                    }
            }
        }
    }
    if constexpr (BLOCK) {
        // A chunk still open at the end (its tail zero-filled) folds too.
        if (((int64_t)T * F_BK) % g.acc_block != 0) {
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) tot[i][j] = __fadd_rn(tot[i][j], acc[i][j]);
        }
    }

#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
        if (m >= g.M) continue;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
            if (n >= g.N) continue;
            double v;
            if constexpr (BLOCK) v = (double)tot[i][j];
            else v = (double)acc[i][j];
            if (g.bias) v = __dadd_rn(v, g.bias[n]);  // Pass.java:202
            g.C[(int64_t)m * g.c_rs + n] = v;
        }
    }
}

// A map of a k-major fp32 operand: dims {rows, K}, row k at k*ld floats,
// 128 x 16 boxes, zero fill outside.
static bool make_map_f32(CUtensorMap *map, const float *Xt, int64_t rows, int64_t ld, int64_t K) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn || ((uintptr_t)Xt % 16) != 0 || (ld % 4) != 0) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)rows, (cuuint64_t)K};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
    const cuuint32_t box[2] = {F_BM, F_BK};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(Xt), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int ORDER>
static int launch_f32(const F32Args &g, const CUtensorMap &ma, const CUtensorMap &mb, dim3 grid,
                      cudaStream_t st) {
    if (cudaFuncSetAttribute(gemm_f32_kernel<ORDER>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             F_SMEM) != cudaSuccess)
        return DRIFT_ECUDA;
    gemm_f32_kernel<ORDER><<<grid, F_THREADS, F_SMEM, st>>>(g, ma, mb);
    return DRIFT_OK;
}

int launch_gemm_f32(Workspace &ws, const drift_policy *p, int64_t M, int64_t N, int64_t K,
                    const double *A, int64_t a_rs, int64_t a_ks, const double *B, int64_t b_rs,
                    int64_t b_ks, const double *bias, double *C, int64_t c_rs, int *d_err,
                    int *d_route, cudaStream_t st, const int **skip) {
    *skip = nullptr;
    const bool order_ok = p->order == DRIFT_SEQUENTIAL || p->order == DRIFT_REVERSED ||
                          (p->order == DRIFT_BLOCKED && std::max<int64_t>(1, p->acc_block) % F_BK == 0);
    if (p->acc != DRIFT_ACC_FP32 || !order_ok || M <= 0 || N <= 0 || K <= 0 ||
        (double)M * (double)N * (double)K < kF32MinMacs || M >= (1LL << 31) ||
        N >= (1LL << 31) || K >= (1LL << 31) || (M + 63) / 64 > 65535)
        return DRIFT_OK;
    const int64_t lda = (M + 3) & ~3LL, ldb = (N + 3) & ~3LL;
    const size_t a_bytes = ((size_t)(K * lda * 4) + 255) & ~(size_t)255;
    const size_t bytes = 256 + a_bytes + (size_t)(K * ldb * 4);
    if (bytes > kF32MaxBytes) return DRIFT_OK;
    char *w = (char *)ws.get(bytes, st);
    if (!w) return DRIFT_OK;  // no room: the double-precision contraction runs alone
    int *props = (int *)w;
    float *At = (float *)(w + 256);
    float *Bt = (float *)(w + 256 + a_bytes);
    CUtensorMap ma, mb;
    memset(&ma, 0, sizeof(ma));
    memset(&mb, 0, sizeof(mb));
    if (!make_map_f32(&ma, At, M, lda, K) || !make_map_f32(&mb, Bt, N, ldb, K)) return DRIFT_OK;

    if (cudaMemsetAsync(props, 0, 64, st) != cudaSuccess) return DRIFT_ECUDA;
    const int grid = sm_count() * 8;
    scan_pack_kernel<<<grid, 256, 0, st>>>(A, M, K, a_rs, a_ks, At, lda, props);
    scan_pack_kernel<<<grid, 256, 0, st>>>(B, N, K, b_rs, b_ks, Bt, ldb, props + kPropWords);
    f32_decide_kernel<<<1, 1, 0, st>>>(props, d_route);

    F32Args g{};
    g.M = M;
    g.N = N;
    g.K = K;
    g.acc_block = std::max<int64_t>(1, p->acc_block);
    g.bias = bias;
    g.C = C;
    g.c_rs = c_rs;
    g.flag = props + kFlagWord;
    g.err = d_err;
    const dim3 fgrid((unsigned)((N + F_BN - 1) / F_BN), (unsigned)((M + F_BM - 1) / F_BM));
    int rc;
    switch (p->order) {
        case DRIFT_SEQUENTIAL: rc = launch_f32<DRIFT_SEQUENTIAL>(g, ma, mb, fgrid, st); break;
        case DRIFT_REVERSED: rc = launch_f32<DRIFT_REVERSED>(g, ma, mb, fgrid, st); break;
        default: rc = launch_f32<DRIFT_BLOCKED>(g, ma, mb, fgrid, st); break;
    }
    if (rc) return rc;
    if (cudaGetLastError() != cudaSuccess) return DRIFT_ECUDA;
    *skip = g.flag;
    return DRIFT_OK;
}

}  // namespace drift
