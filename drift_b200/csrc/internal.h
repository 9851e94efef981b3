// internal.h — declarations shared by the engine's translation units.
#pragma once

#include <cstdint>
#include <map>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/drift_b200.h"

namespace drift {

// A growable device scratch buffer, allocated and freed in stream order.
// Every call through one context shares it, so calls on different streams
// of the same context must not overlap.
class Workspace {
   public:
    void *get(size_t bytes, cudaStream_t st);
    void release(cudaStream_t st);

   private:
    void *ptr_ = nullptr;
    size_t cap_ = 0;
};

// Device copies of Dot.pairwise leaf schedules, one per K, kept for the
// life of the context.
class ScheduleCache {
   public:
    const uint8_t *get(int64_t K, cudaStream_t st);
    int64_t leaves(int64_t K) const;
    int last_status() const { return status_; }
    void clear();

   private:
    struct Entry {
        uint8_t *d;
        int64_t leaves;
    };
    std::map<int64_t, Entry> entries_;
    int status_ = DRIFT_OK;
};

int pairwise_schedule(int64_t K, std::vector<uint8_t> &sched, int *depth);

int launch_amax(const double *d_x, int64_t n, double *d_amax, cudaStream_t st);
int launch_per_tensor_scale(int fmt, const double *d_amax, double *d_scale, cudaStream_t st);
// The number of Rng draws a stochastic cast of d_src[0..n) would take
// (0 for any other rounding), written to *d_draws.
int launch_quantize_draws(Workspace &ws, const drift_policy *p, int fmt, int rm,
                          const double *d_src, int64_t n, const double *d_scale, double scale,
                          uint64_t *d_draws, int *d_err, cudaStream_t st);
// `rows` tensors of `len` elements cast one by one, each with its own
// per-tensor scale; clamps added per row. Nearest-even or truncate, no MX.
int launch_quantize_rows(const drift_policy *p, int fmt, int rm, const double *d_src,
                         double *d_dst, int64_t rows, int64_t len,
                         unsigned long long *d_clamped, int *d_err, cudaStream_t st);
int launch_quantize(Workspace &ws, const drift_policy *p, int fmt, int rm, const double *d_src,
                    double *d_dst, int64_t n, const double *d_scale, double scale,
                    uint64_t *d_state, unsigned long long *d_clamped, int *d_err,
                    cudaStream_t st);
int launch_quantize_noalloc(const drift_policy *p, int fmt, int rm, const double *d_src,
                            double *d_dst, int64_t n, const double *d_scale, double scale,
                            uint64_t *d_state, unsigned long long *d_clamped, int *d_err,
                            cudaStream_t st);
int launch_encode(Workspace &ws, int fmt, int rm, const double *d_v, int32_t *d_codes, int64_t n,
                  uint64_t *d_state, int *d_err, cudaStream_t st);
int launch_decode(int fmt, const int32_t *d_codes, double *d_v, int64_t n, cudaStream_t st);
int launch_acc_round(Workspace &ws, int acc, int rm, const double *d_x, double *d_y, int64_t n,
                     uint64_t *d_state, int *d_err, cudaStream_t st);
int launch_error_sums(const double *got, const double *exact, int64_t n, double *sums,
                      cudaStream_t st);
int launch_radix_pass(const double *got, const double *exact, int64_t n, int pass,
                      unsigned long long *state, unsigned long long *hist, cudaStream_t st);
int launch_group_kth(const double *got, const double *exact, int64_t groups, int64_t n,
                     int64_t k, double *out, cudaStream_t st);
int launch_radix_select(int pass, const unsigned long long *hist, unsigned long long *state,
                        cudaStream_t st);
// contract.cu: a contraction with its buffers (a, b, c before the op's
// offsets) and an optional bias of `cols` values (drift_gemm's linears).
struct ContractDesc {
    drift_contraction op;
    const double *a;
    const double *b;
    double *c;
    const double *bias;
};
int check_contraction(const drift_contraction &op);
// A FULL-window, non-stochastic contraction with one output per thread and
// the operands staged in shared memory (contract.cu): the launch for calls
// whose outputs are too few for the tiled kernel to fill the GPU. It stands
// down at once if `skip` is given and reads nonzero; `route`, when given,
// receives DRIFT_ROUTE_STAGED.
int launch_contract_staged(const drift_policy *p, const ContractDesc &d, const int *skip,
                           int *route, cudaStream_t st);
// The default thin-call limit of a policy: GEMMs with fewer 64 x 64 output
// tiles run on launch_contract_staged.
int64_t staged_tile_limit(const drift_policy *p);
int launch_contract(Workspace &ws, ScheduleCache &cache, const drift_policy *p,
                    const ContractDesc &d, uint64_t *d_state, int *d_err, cudaStream_t st);
// A batch of `batch` contractions, problem z at A + z*a_bs, B + z*b_bs,
// C + z*c_bs (element strides), all with the same shape and bias.
int launch_gemm_batched(Workspace &ws, ScheduleCache &cache, const drift_policy *p, int64_t batch,
                        int64_t M, int64_t N, int64_t K, const double *A, int64_t a_rs,
                        int64_t a_ks, int64_t a_bs, const double *B, int64_t b_rs, int64_t b_ks,
                        int64_t b_bs, const double *bias, double *C, int64_t c_rs, int64_t c_bs,
                        int *d_err, cudaStream_t st);
int launch_fp64_probe(cudaStream_t st, double *ops_per_s);
int launch_fp32_probe(cudaStream_t st, double *fma_per_s);
// One contraction C = A B^T (+ bias). `d_route`, when given, receives the
// DRIFT_ROUTE_* of the path taken. `d_scan` (8 device words), when given,
// lets FP32 and BF16 accumulators scan their operands for the range proof
// that drops the per-step checks. `*n_launched` receives the number of
// kernels queued.
// Calls with fewer 64 x 64 output tiles than `thin_tiles` run one output per
// thread (launch_contract_staged); a negative value means two per SM.
int launch_gemm(Workspace &ws, ScheduleCache &cache, const drift_policy *p, int64_t M, int64_t N,
                int64_t K, const double *A, int64_t a_rs, int64_t a_ks, const double *B,
                int64_t b_rs, int64_t b_ks, const double *bias, double *C, int64_t c_rs,
                int64_t thin_tiles, int *d_err, int *d_route, cudaStream_t st,
                unsigned *d_scan = nullptr, int *n_launched = nullptr);
// gemm32.cu: queues the FP32-pipe path of an FP32-accumulated contraction
// whose policy and shape qualify (an operand scan, a device-side decision and
// the FFMA contraction, which stands down unless the scan allows it). Sets
// *skip to the decision word the double-precision contraction must then
// check, or leaves it null when the path does not apply to this call. Uses
// `ws` for the scan and the transposed operands.
int launch_gemm_f32(Workspace &ws, const drift_policy *p, int64_t M, int64_t N, int64_t K,
                    const double *A, int64_t a_rs, int64_t a_ks, const double *B, int64_t b_rs,
                    int64_t b_ks, const double *bias, double *C, int64_t c_rs, int *d_err,
                    int *d_route, cudaStream_t st, const int **skip);

// tables.cu
int launch_value_table(int fmt, uint64_t *d_bits, cudaStream_t st);
int launch_pair_table(int fmt, int mode, uint64_t seed, int64_t first, int64_t n, int32_t *d_a,
                      int32_t *d_b, int32_t *d_prod, int32_t *d_sum, cudaStream_t st);

// train.cu
int launch_embed_gather(const int32_t *tokens, int64_t n_tok, const double *table, int64_t vocab,
                        int64_t width, double *out, int *err, cudaStream_t st);
int launch_embed_grad(const int32_t *tokens, int64_t n_tok, const double *rows, int64_t width,
                      double *grad, int64_t vocab, cudaStream_t st);
int launch_bias_grad(const double *dy, int64_t rows, int64_t cols, double *db, cudaStream_t st);
int launch_tanh_backward(const double *out, double *grad, int64_t n, cudaStream_t st);
int launch_scale_for(int fmt, const double *amax_now, double *hist, int32_t len, int64_t *count,
                     double *scale, cudaStream_t st);
int launch_adam(double *p, const double *g, double *m, double *v, int64_t n, double c1, double c2,
                double lr, int fp32, cudaStream_t st);

// Streaming multiprocessors of the current device (148 on B200), used to size
// grid-stride launches; 148 if the query fails.
inline int sm_count() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        sms <= 0)
        return 148;
    return sms;
}

}  // namespace drift
