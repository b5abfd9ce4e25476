// The language-model head with its cross-entropy loss, fused (model.py:153-157):
//   loss = mean over rows r with targets[r] != -1 of (logsumexp(h_r W^T) - (h_r W^T)[targets[r]])
// The (N x V) logits are never written. Forward: one tensor-core product whose epilogue keeps, per
// row and column block, the running max and sum of exponentials (EPI_LSE) and picks up the target's
// logit; a small kernel combines the blocks into the row's logsumexp and the mean loss.
// Backward: the same product again, its epilogue writing dlogits = (softmax - onehot) * dloss / count
// in the operand type (EPI_CE_GRAD), then dh = dlogits W and dW = dlogits^T h.
#include "gemm.cuh"

namespace ulm {
namespace {

constexpr int HEAD_LOSS_THREADS = 256;

// column blocks of the EPI_LSE partials: the narrowest block of any back end is 64 columns
int64_t head_part_ld(int64_t V) { return cdiv(V, 64); }

struct HeadWork {
  float* part;      // N x part_ld x 2 (max, sum exp)
  float* tgt;       // N target logits
  float* row_loss;  // ctas partial sums of the row losses
  int* row_count;   // ctas partial counts of the rows that count
  float* scale;     // dloss / count (backward)
  void* dlogits;    // N x ld_v in the operand type (backward)
  int64_t bytes;
};

inline int64_t al256h(int64_t n) { return (n + 255) / 256 * 256; }

HeadWork carve_head(void* base, int64_t N, int64_t V, int dt) {
  HeadWork w;
  char* p = static_cast<char*>(base);
  char* p0 = p;
  auto take = [&](int64_t bytes) {
    char* q = p;
    p += al256h(bytes);
    return q;
  };
  const int64_t ctas = cdiv(N, HEAD_LOSS_THREADS / 32);  // the loss kernel's CTAs (one row per warp)
  w.part = reinterpret_cast<float*>(take(N * head_part_ld(V) * 2 * 4));
  w.tgt = reinterpret_cast<float*>(take(N * 4));
  w.row_loss = reinterpret_cast<float*>(take(ctas * 4));
  w.row_count = reinterpret_cast<int*>(take(ctas * 4));
  w.scale = reinterpret_cast<float*>(take(4));
  w.dlogits = take(N * ulm_operand_ld(V) * (dt == ULM_F32 ? 4 : 2));
  w.bytes = p - p0;
  return w;
}

// per row: lse = M + log(sum_j s_j exp(m_j - M)) over the column blocks that hold logits (s_j > 0),
// the row's loss lse - target logit (when its target is not -1); one warp per row (its lanes read
// the row's (max, sum) pairs side by side), per CTA partial sums of its HEAD_ROWS rows in row order
constexpr int HEAD_ROWS = HEAD_LOSS_THREADS / 32;
__global__ void __launch_bounds__(HEAD_LOSS_THREADS)
    head_lse_kernel(const float* __restrict__ part, int64_t part_ld, const float* __restrict__ tgt_logit,
                    const int64_t* __restrict__ targets, float* __restrict__ lse, float* __restrict__ row_loss,
                    int* __restrict__ row_count, int64_t N) {
  __shared__ float lred[HEAD_ROWS];
  __shared__ int cred[HEAD_ROWS];
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const int64_t r = (int64_t)blockIdx.x * HEAD_ROWS + wp;
  float loss = 0.f;
  int cnt = 0;
  if (r < N) {
    const float2* pp = reinterpret_cast<const float2*>(part + r * part_ld * 2);
    float M = -INFINITY;
    for (int64_t j = lane; j < part_ld; j += 32) {
      const float2 e = pp[j];
      if (e.y > 0.f) M = fmaxf(M, e.x);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float s = 0.f;
    for (int64_t j = lane; j < part_ld; j += 32) {
      const float2 e = pp[j];
      if (e.y > 0.f) s += e.y * expf(e.x - M);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float l = M + logf(s);
    if (lane == 0) lse[r] = l;
    if (targets[r] >= 0) {
      loss = l - tgt_logit[r];
      cnt = 1;
    }
  }
  if (lane == 0) {
    lred[wp] = loss;
    cred[wp] = cnt;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float ls = 0.f;
    int cs = 0;
    for (int i = 0; i < HEAD_ROWS; ++i) {
      ls += lred[i];
      cs += cred[i];
    }
    row_loss[blockIdx.x] = ls;
    row_count[blockIdx.x] = cs;
  }
}

// loss = sum of the CTA partials / count (in order, double accumulation); count kept for the backward
__global__ void head_loss_kernel(const float* __restrict__ row_loss, const int* __restrict__ row_count, int64_t ctas,
                                 float* __restrict__ loss, float* __restrict__ count_out) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  double s = 0.0;
  long long c = 0;
  for (int64_t i = 0; i < ctas; ++i) {
    s += row_loss[i];
    c += row_count[i];
  }
  *loss = c > 0 ? (float)(s / (double)c) : NAN;  // F.cross_entropy's mean over no rows is nan
  *count_out = (float)c;
}

__global__ void head_scale_kernel(const float* __restrict__ dloss, const float* __restrict__ count,
                                  float* __restrict__ scale) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *scale = *count > 0.f ? *dloss / *count : 0.f;
}

int head_check(const void* h_op, int64_t ld_h, const void* w_op, int64_t ld_w, const int64_t* targets, int64_t N,
               int64_t V, int64_t D, int prec) {
  ULM_REQUIRE(prec == ULM_PREC_BF16 || prec == ULM_PREC_FP32, "prec must be ULM_PREC_BF16 or ULM_PREC_FP32");
  ULM_REQUIRE(h_op && w_op && targets, "null pointer argument");
  ULM_REQUIRE(N > 0 && V > 0 && D > 0, "bad extents");
  ULM_REQUIRE(N < (1ll << 31) && V < (1 << 30) && D < (1 << 30), "extent too large");
  ULM_REQUIRE(ld_h >= D && ld_w >= D, "row stride shorter than the row");
  return ULM_OK;
}

}  // namespace
}  // namespace ulm

using namespace ulm;

extern "C" int64_t ulm_lm_head_work_bytes(int64_t N, int64_t V, int64_t D, int prec) {
  if (N < 0 || V < 0 || D < 0) return -1;
  return carve_head(nullptr, N, V, prec == ULM_PREC_FP32 ? ULM_F32 : ULM_BF16).bytes;
}

extern "C" int ulm_lm_head_loss_fwd(const void* h_op, int64_t ld_h, const void* w_op, int64_t ld_w,
                                    const int64_t* targets, float* lse, float* loss, float* count, void* work,
                                    int64_t N, int64_t V, int64_t D, int prec, void* stream) {
  if (int rc = head_check(h_op, ld_h, w_op, ld_w, targets, N, V, D, prec)) return rc;
  ULM_REQUIRE(lse && loss && count && work, "null pointer argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int dt = prec == ULM_PREC_FP32 ? ULM_F32 : ULM_BF16;
  HeadWork hw = carve_head(work, N, V, dt);
  const int64_t pld = head_part_ld(V);
  ULM_CUDA_TRY(cudaMemsetAsync(hw.part, 0, N * pld * 2 * sizeof(float), st));
  ULM_CUDA_TRY(cudaMemsetAsync(hw.tgt, 0, N * sizeof(float), st));
  // logits = h W^T: A = h (rows, K-major), B = W (classes, K-major); only the epilogue's partials
  Operand A{h_op, ld_h, N * ld_h, D, N, dt, false};
  Operand Bw{w_op, ld_w, V * ld_w, D, V, dt, false};
  GemmShape s{1, (int)N, (int)V, (int)D, CAUSAL_NONE};
  GemmEpilogue e;
  e.kind = EPI_LSE;
  e.out_dtype = ULM_F32;
  e.out = nullptr;
  e.ldo = V;
  e.out_bstride = N * V;
  e.g = nullptr;
  e.vec_ok = 0;
  e.aux = nullptr;
  e.ld_aux = 0;
  e.aux_bstride = 0;
  e.tile_partial = hw.tgt;
  e.row_partial = hw.part;
  e.part_ld = (int)pld;
  e.staged = 0;
  e.targets = targets;
  e.rows_valid = (int)N;
  if (int rc = run_gemm(A, Bw, s, e, st)) return rc;
  const int64_t ctas = cdiv(N, HEAD_ROWS);
  head_lse_kernel<<<(unsigned)ctas, HEAD_LOSS_THREADS, 0, st>>>(hw.part, pld, hw.tgt, targets, lse, hw.row_loss,
                                                                hw.row_count, N);
  ULM_LAUNCH_CHECK("head_lse_kernel");
  head_loss_kernel<<<1, 32, 0, st>>>(hw.row_loss, hw.row_count, ctas, loss, count);
  ULM_LAUNCH_CHECK("head_loss_kernel");
  return ULM_OK;
}

extern "C" int ulm_lm_head_loss_bwd(const float* dloss, const float* count, const void* h_op, int64_t ld_h,
                                    const void* w_op, int64_t ld_w, const int64_t* targets, const float* lse,
                                    float* dh, float* dw, void* work, int64_t N, int64_t V, int64_t D, int prec,
                                    void* stream) {
  if (int rc = head_check(h_op, ld_h, w_op, ld_w, targets, N, V, D, prec)) return rc;
  ULM_REQUIRE(dloss && count && lse && dh && dw && work, "null pointer argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int dt = prec == ULM_PREC_FP32 ? ULM_F32 : ULM_BF16;
  HeadWork hw = carve_head(work, N, V, dt);
  const int64_t ldv = ulm_operand_ld(V);
  head_scale_kernel<<<1, 32, 0, st>>>(dloss, count, hw.scale);
  ULM_LAUNCH_CHECK("head_scale_kernel");
  {
    // dlogits = (softmax - onehot) * dloss / count, recomputing the logits
    Operand A{h_op, ld_h, N * ld_h, D, N, dt, false};
    Operand Bw{w_op, ld_w, V * ld_w, D, V, dt, false};
    GemmShape s{1, (int)N, (int)V, (int)D, CAUSAL_NONE};
    GemmEpilogue e = make_epilogue(EPI_CE_GRAD, dt, hw.dlogits, ldv, N * ldv, nullptr);
    e.targets = targets;
    e.row_lse = lse;
    e.scale = hw.scale;
    e.rows_valid = (int)N;
    if (int rc = run_gemm(A, Bw, s, e, st)) return rc;
  }
  {
    // dh = dlogits W: A = dlogits (rows, K-major over classes), B = W as [class][d] (MN-major)
    Operand A{hw.dlogits, ldv, N * ldv, V, N, dt, false};
    Operand Bw{w_op, ld_w, V * ld_w, D, V, dt, true};
    GemmShape s{1, (int)N, (int)D, (int)V, CAUSAL_NONE};
    GemmEpilogue e = make_epilogue(EPI_STORE, ULM_F32, dh, D, N * D, nullptr);
    if (int rc = run_gemm(A, Bw, s, e, st)) return rc;
  }
  {
    // dW = dlogits^T h: A = dlogits as [row][class] (MN-major), B = h as [row][d] (MN-major)
    Operand A{hw.dlogits, ldv, N * ldv, V, N, dt, true};
    Operand Bh{h_op, ld_h, N * ld_h, D, N, dt, true};
    GemmShape s{1, (int)V, (int)D, (int)N, CAUSAL_NONE};
    GemmEpilogue e = make_epilogue(EPI_STORE, ULM_F32, dw, D, V * D, nullptr);
    if (int rc = run_gemm(A, Bh, s, e, st)) return rc;
  }
  return ULM_OK;
}
