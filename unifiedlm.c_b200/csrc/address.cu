// The addressing prologue of UnifiedBlock (model.py:61-62, 70-72, 79) and its backward:
//
//   u = causal depthwise conv(h)                   (width K, oldest -> newest weights)
//   a = u K^T + b,  z = relu(a)^2                  (key GEMM on the tensor cores, fused epilogue)
//   r = z / den,  den = eps + sum_m z              (row normalisation)
//
// Backward, with dr the gradient reaching r (from the fast memory's statistics backward):
//   s = sum_m dr_m r_m,  dz = (dr - s) / den,  da = 2 sqrt(z) dz  (relu(a) = sqrt(z) where a > 0)
//   d eps = -sum_rows s / den,  db = sum_rows da,  dK = da^T u,  du = da K
//   dh[t] = sum_j conv[j] du[t + K-1-j],  dconv[j] = sum_{b,t} du[t] h[t - K+1+j]
// The contractions run on the GEMM engine (gemm.cu): tcgen05 with bf16 operands, or fp32 FMA in the
// fp32 parity mode. Column sums (db, dconv) go through per-CTA partials reduced in a fixed order.
#include <algorithm>

#include "gemm.cuh"

namespace ulm {

template <typename T>
__device__ __forceinline__ float ld_as_float(const void* p, int64_t i);
template <>
__device__ __forceinline__ float ld_as_float<float>(const void* p, int64_t i) {
  return static_cast<const float*>(p)[i];
}
template <>
__device__ __forceinline__ float ld_as_float<__nv_bfloat16>(const void* p, int64_t i) {
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ void st_as(void* p, int64_t i, float v, int dt) {
  if (dt == ULM_F32)
    static_cast<float*>(p)[i] = v;
  else
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

// u[b,t,d] = sum_j conv_w[d, j] * h[b, t-K+1+j, d] (zero before the sequence start)
template <typename InT>
__global__ void addr_conv_kernel(const void* __restrict__ h, const float* __restrict__ conv_w, void* __restrict__ u,
                                 int u_dtype, int64_t ld_u, int T, int D, int K, int64_t rows) {
  const int64_t n = rows * D;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / D;
    const int d = (int)(i - row * D);
    const int t = (int)(row % T);
    float acc = 0.f;
    for (int j = 0; j < K; ++j) {
      const int tt = t - K + 1 + j;
      if (tt >= 0) acc = fmaf(conv_w[d * K + j], ld_as_float<InT>(h, (row - t + tt) * D + d), acc);
    }
    st_as(u, row * ld_u + d, acc, u_dtype);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// r = z / (eps + sum z) in place, one warp per row; den saved for the backward
__global__ void addr_normalize_kernel(float* __restrict__ zr, float* __restrict__ den, const float* __restrict__ eps,
                                      int64_t rows, int M) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float* z = zr + row * M;
  float s = 0.f;
  for (int m = lane; m < M; m += 32) s += z[m];
  s = warp_sum(s);
  const float dn = *eps + s;
  for (int m = lane; m < M; m += 32) z[m] = z[m] / dn;
  if (lane == 0) den[row] = dn;
}

// one warp per row: s = sum dr r, da = 2 sqrt(r den) (dr - s) / den; the CTA also sums da over its
// rows per column (db partial) and -s/den over its rows (d eps partial)
template <int WARPS>
__global__ void __launch_bounds__(32 * WARPS)
    addr_bwd_kernel(const float* __restrict__ dr, const float* __restrict__ r, const float* __restrict__ den,
                    void* __restrict__ da, int da_dtype, int64_t ld_da, float* __restrict__ db_part,
                    float* __restrict__ deps_part, int64_t rows, int M, int rows_per_cta) {
  extern __shared__ float col_acc[];  // [WARPS][M]
  __shared__ float deps_w[WARPS];
  const int wp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int m = threadIdx.x; m < WARPS * M; m += blockDim.x) col_acc[m] = 0.f;
  __syncthreads();
  float deps_acc = 0.f;
  const int64_t row0 = (int64_t)blockIdx.x * rows_per_cta;
  for (int rr = wp; rr < rows_per_cta; rr += WARPS) {
    const int64_t row = row0 + rr;
    if (row >= rows) break;
    const float* drr = dr + row * M;
    const float* rrow = r + row * M;
    float s = 0.f;
    for (int m = lane; m < M; m += 32) s = fmaf(drr[m], rrow[m], s);
    s = warp_sum(s);
    const float dn = den[row];
    const float inv = 1.0f / dn;
    deps_acc -= s * inv;
    float* acc = col_acc + wp * M;
    for (int m = lane; m < M; m += 32) {
      const float rv = rrow[m];
      const float dav = 2.f * sqrtf(rv * dn) * ((drr[m] - s) * inv);
      st_as(da, row * ld_da + m, dav, da_dtype);
      acc[m] += dav;
    }
  }
  if (lane == 0) deps_w[wp] = deps_acc;
  __syncthreads();
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    float t = 0.f;
    for (int w = 0; w < WARPS; ++w) t += col_acc[w * M + m];
    db_part[(int64_t)blockIdx.x * M + m] = t;
  }
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < WARPS; ++w) t += deps_w[w];
    deps_part[blockIdx.x] = t;
  }
}

// out[i] = sum_p part[p][i] over nparts, in order (dK from the split-K partials, db)
__global__ void sum_parts_kernel(const float* __restrict__ part, int64_t nparts, int64_t n, float* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int64_t p = 0; p < nparts; ++p) s += part[p * n + i];
    out[i] = s;
  }
}

// deterministic sum of n floats into *out (one block)
__global__ void __launch_bounds__(256) sum_all_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ out) {
  __shared__ double red[256];
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < n; i += 256) s += x[i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int st = 128; st > 0; st >>= 1) {
    if ((int)threadIdx.x < st) red[threadIdx.x] += red[threadIdx.x + st];
    __syncthreads();
  }
  if (threadIdx.x == 0) *out = (float)red[0];
}

// dh and the conv-weight partials. CTA = 32 channels x 8 time lanes over a chunk of positions of one
// batch row; dconv partial per (chunk, b) reduced later.
template <typename InT>
__global__ void __launch_bounds__(256)
    addr_conv_bwd_kernel(const float* __restrict__ du, const void* __restrict__ h, const float* __restrict__ conv_w,
                         float* __restrict__ dh, float* __restrict__ dconv_part, int T, int D, int K, int t_chunk) {
  __shared__ float red[8][32][8];  // [time lane][channel][tap], K <= 8
  const int lane = threadIdx.x & 31, tl = threadIdx.x >> 5;
  const int d = blockIdx.x * 32 + lane;
  const int b = blockIdx.y;
  const int t0 = blockIdx.z * t_chunk, t1 = min(T, t0 + t_chunk);
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  if (d < D) {
    const int64_t base = (int64_t)b * T;
    for (int t = t0 + tl; t < t1; t += 8) {
      float g = 0.f;
      for (int j = 0; j < K; ++j) {
        const int tt = t + K - 1 - j;  // output position that used h[t] through tap j
        if (tt < T) g = fmaf(conv_w[d * K + j], du[(base + tt) * D + d], g);
      }
      dh[(base + t) * D + d] = g;
      const float dut = du[(base + t) * D + d];
      for (int j = 0; j < K; ++j) {
        const int ts = t - K + 1 + j;
        if (ts >= 0) acc[j] = fmaf(dut, ld_as_float<InT>(h, (base + ts) * D + d), acc[j]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[tl][lane][j] = acc[j];
  __syncthreads();
  if (tl == 0 && d < D) {
    const int64_t part = (int64_t)blockIdx.z * gridDim.y + blockIdx.y;
    for (int j = 0; j < K; ++j) {
      float s = 0.f;
      for (int l = 0; l < 8; ++l) s += red[l][lane][j];
      dconv_part[(part * D + d) * K + j] = s;
    }
  }
}

GemmEpilogue plain_epilogue(int kind, int out_dtype, void* out, int64_t ldo, int64_t bstride) {
  GemmEpilogue e;
  e.kind = kind;
  e.out_dtype = out_dtype;
  e.out = out;
  e.ldo = ldo;
  e.out_bstride = bstride;
  e.g = nullptr;
  e.aux = nullptr;
  e.ld_aux = 0;
  e.aux_bstride = 0;
  e.tile_partial = nullptr;
  const int vec = out_dtype == ULM_F32 ? 4 : 8;
  e.vec_ok = is_aligned16(out) && ldo % vec == 0 && bstride % vec == 0;
  return e;
}

struct AddrBwdWork {
  void* da;         // rows x ld_m, op dtype
  float* du;        // rows x D
  float* dk_part;   // S x M x D
  float* db_part;   // ctas x M
  float* deps_part; // ctas
  float* dconv_part;
  int64_t ld_m;
  int S, ctas, chunks;
  int64_t bytes;
};

constexpr int ADDR_ROWS_PER_CTA = 64;
constexpr int ADDR_CONV_CHUNK = 64;

inline int64_t al256(int64_t n) { return (n + 255) / 256 * 256; }

inline int addr_split(int64_t rows) {
  // split the B*T contraction of dK into S chunks so the product has enough tiles
  for (int s = 8; s > 1; s /= 2)
    if (rows % s == 0 && rows / s >= 256) return s;
  return 1;
}

inline AddrBwdWork carve_addr_work(void* base, int64_t B, int64_t T, int64_t D, int64_t M, int op_dt) {
  AddrBwdWork w;
  const int64_t rows = B * T;
  w.ld_m = ulm_operand_ld(M);
  w.S = addr_split(rows);
  w.ctas = (int)cdiv(rows, ADDR_ROWS_PER_CTA);
  w.chunks = (int)cdiv(T, ADDR_CONV_CHUNK);
  char* p = static_cast<char*>(base);
  char* p0 = p;
  auto take = [&](int64_t bytes) {
    char* q = p;
    p += al256(bytes);
    return q;
  };
  w.da = take(rows * w.ld_m * (op_dt == ULM_F32 ? 4 : 2));
  w.du = reinterpret_cast<float*>(take(rows * D * 4));
  w.dk_part = reinterpret_cast<float*>(take((int64_t)w.S * M * D * 4));
  w.db_part = reinterpret_cast<float*>(take((int64_t)w.ctas * M * 4));
  w.deps_part = reinterpret_cast<float*>(take((int64_t)w.ctas * 4));
  w.dconv_part = reinterpret_cast<float*>(take((int64_t)w.chunks * B * D * 8 * 4));
  w.bytes = p - p0;
  return w;
}

}  // namespace ulm

using namespace ulm;

namespace {

int addr_check(int h_dtype, int prec, int64_t B, int64_t T, int64_t D, int64_t M, int64_t K) {
  ULM_REQUIRE(h_dtype == ULM_F32 || h_dtype == ULM_BF16, "h_dtype must be ULM_F32 or ULM_BF16");
  ULM_REQUIRE(prec == ULM_PREC_BF16 || prec == ULM_PREC_FP32, "bad prec");
  ULM_REQUIRE(B > 0 && T > 0 && D > 0 && M > 0, "empty problem");
  ULM_REQUIRE(K >= 1 && K <= 8, "conv_size must be in [1, 8]");
  ULM_REQUIRE(B * T < (1ll << 31) && M < (1 << 30) && D < (1 << 30), "extent too large");
  return ULM_OK;
}

}  // namespace

extern "C" int ulm_address_fwd(const void* h, int h_dtype, const float* conv_w, int64_t conv_size, const void* key_w,
                               int64_t ld_kw, const float* key_b, const float* eps, float* r, float* den, void* u_op,
                               int64_t ld_u, int64_t B, int64_t T, int64_t D, int64_t M, int prec, void* stream) {
  if (int rc = addr_check(h_dtype, prec, B, T, D, M, conv_size)) return rc;
  ULM_REQUIRE(h && conv_w && key_w && key_b && eps && r && den && u_op, "null pointer argument");
  ULM_REQUIRE(ld_u >= D && ld_kw >= D, "row stride shorter than the row");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int dt = prec == ULM_PREC_FP32 ? ULM_F32 : ULM_BF16;
  const int64_t rows = B * T;
  const unsigned grid = (unsigned)std::min<int64_t>(cdiv(rows * D, 256), 16 * 148);
  if (h_dtype == ULM_F32)
    addr_conv_kernel<float><<<grid, 256, 0, st>>>(h, conv_w, u_op, dt, ld_u, (int)T, (int)D, (int)conv_size, rows);
  else
    addr_conv_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(h, conv_w, u_op, dt, ld_u, (int)T, (int)D, (int)conv_size,
                                                          rows);
  ULM_LAUNCH_CHECK("addr_conv_kernel");
  // z = relu(u K^T + b)^2 written into r
  Operand A{u_op, ld_u, rows * ld_u, D, rows, dt, false};
  Operand Bw{key_w, ld_kw, M * ld_kw, D, M, dt, false};
  GemmShape s{1, (int)rows, (int)M, (int)D, CAUSAL_NONE};
  GemmEpilogue e = plain_epilogue(EPI_RELU2, ULM_F32, r, M, rows * M);
  e.aux = key_b;
  if (int rc = run_gemm(A, Bw, s, e, st)) return rc;
  addr_normalize_kernel<<<(unsigned)cdiv(rows, 8), 256, 0, st>>>(r, den, eps, rows, (int)M);
  ULM_LAUNCH_CHECK("addr_normalize_kernel");
  return ULM_OK;
}

extern "C" int64_t ulm_address_bwd_work_bytes(int64_t B, int64_t T, int64_t D, int64_t M, int prec) {
  return carve_addr_work(nullptr, B, T, D, M, prec == ULM_PREC_FP32 ? ULM_F32 : ULM_BF16).bytes;
}

extern "C" int ulm_address_bwd(const float* dr, const float* r, const float* den, const void* u_op, int64_t ld_u,
                               const void* h, int h_dtype, const float* conv_w, int64_t conv_size, const void* key_w,
                               int64_t ld_kw, float* dh, float* dconv_w, float* dkey_w, float* dkey_b, float* deps,
                               void* work, int64_t B, int64_t T, int64_t D, int64_t M, int prec, void* stream) {
  if (int rc = addr_check(h_dtype, prec, B, T, D, M, conv_size)) return rc;
  ULM_REQUIRE(dr && r && den && u_op && h && conv_w && key_w && dh && dconv_w && dkey_w && dkey_b && deps && work,
              "null pointer argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int dt = prec == ULM_PREC_FP32 ? ULM_F32 : ULM_BF16;
  const int64_t rows = B * T;
  AddrBwdWork wk = carve_addr_work(work, B, T, D, M, dt);
  // da, and the db / d eps partials
  constexpr int W = 8;
  const size_t smem = (size_t)W * M * sizeof(float);
  ULM_REQUIRE(smem <= 200 * 1024, "M too large for the addressing backward (M <= 6400)");
  ULM_CUDA_TRY(cudaFuncSetAttribute(addr_bwd_kernel<W>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  addr_bwd_kernel<W><<<(unsigned)wk.ctas, 32 * W, smem, st>>>(dr, r, den, wk.da, dt, wk.ld_m, wk.db_part,
                                                              wk.deps_part, rows, (int)M, ADDR_ROWS_PER_CTA);
  ULM_LAUNCH_CHECK("addr_bwd_kernel");
  sum_parts_kernel<<<(unsigned)cdiv(M, 256), 256, 0, st>>>(wk.db_part, wk.ctas, M, dkey_b);
  ULM_LAUNCH_CHECK("sum_parts_kernel");
  sum_all_kernel<<<1, 256, 0, st>>>(wk.deps_part, wk.ctas, deps);
  ULM_LAUNCH_CHECK("sum_all_kernel");
  // dK = da^T u, split over S chunks of rows (each chunk a GEMM batch), then summed in order
  {
    const int64_t rc_rows = rows / wk.S;
    Operand A{wk.da, wk.ld_m, rc_rows * wk.ld_m, M, rc_rows, dt, true};
    Operand Bu{u_op, ld_u, rc_rows * ld_u, D, rc_rows, dt, true};
    GemmShape s{wk.S, (int)M, (int)D, (int)rc_rows, CAUSAL_NONE};
    GemmEpilogue e = plain_epilogue(EPI_STORE, ULM_F32, wk.dk_part, D, M * D);
    if (int rc = run_gemm(A, Bu, s, e, st)) return rc;
    sum_parts_kernel<<<(unsigned)std::min<int64_t>(cdiv(M * D, 256), 16 * 148), 256, 0, st>>>(wk.dk_part, wk.S,
                                                                                              M * D, dkey_w);
    ULM_LAUNCH_CHECK("sum_parts_kernel");
  }
  // du = da K
  {
    Operand A{wk.da, wk.ld_m, rows * wk.ld_m, M, rows, dt, false};
    Operand Bw{key_w, ld_kw, M * ld_kw, D, M, dt, true};
    GemmShape s{1, (int)rows, (int)D, (int)M, CAUSAL_NONE};
    GemmEpilogue e = plain_epilogue(EPI_STORE, ULM_F32, wk.du, D, rows * D);
    if (int rc = run_gemm(A, Bw, s, e, st)) return rc;
  }
  // through the conv
  dim3 grid((unsigned)cdiv(D, 32), (unsigned)B, (unsigned)wk.chunks);
  if (h_dtype == ULM_F32)
    addr_conv_bwd_kernel<float><<<grid, 256, 0, st>>>(wk.du, h, conv_w, dh, wk.dconv_part, (int)T, (int)D,
                                                       (int)conv_size, ADDR_CONV_CHUNK);
  else
    addr_conv_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(wk.du, h, conv_w, dh, wk.dconv_part, (int)T, (int)D,
                                                               (int)conv_size, ADDR_CONV_CHUNK);
  ULM_LAUNCH_CHECK("addr_conv_bwd_kernel");
  sum_parts_kernel<<<(unsigned)cdiv(D * conv_size, 256), 256, 0, st>>>(wk.dconv_part, (int64_t)wk.chunks * B,
                                                                       D * conv_size, dconv_w);
  ULM_LAUNCH_CHECK("sum_parts_kernel");
  return ULM_OK;
}
