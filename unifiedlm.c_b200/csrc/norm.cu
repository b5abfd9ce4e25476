// RMSNorm and the plain Linear of UnifiedBlock's input side (the reference's RMSNorm, model.py:31-42,
// and `val`, model.py:65, 81), so the whole block runs in this library.
//
// RMSNorm: one warp per row (columns strided over the lanes, coalesced), fp32 statistics:
//   xh = x * rstd, rstd = 1 / sqrt(mean(x^2) + eps), y = round_x(xh) * weight
// where round_x is the rounding to x's type (the reference's `.type_as(x)` before the weight).
// Backward: dxh = dy * weight, dx = rstd * (dxh - xh * mean(dxh * xh)); dweight = sum over rows of
// dy * round_x(xh), per-CTA partial rows summed in a fixed order.
//
// Linear: y = x W^T on the batched GEMM engine (bf16 operands on the tensor cores with fp32
// accumulation, or the fp32 FMA back end), dx = dy W, dW = dy^T x (split K over the rows, partials
// summed in a fixed order).
#include "gemm.cuh"

namespace ulm {
namespace {

constexpr int NORM_WARPS = 8;  // rows per CTA

__device__ __forceinline__ float load_as_float(const void* p, int dt, int64_t i) {
  return dt == ULM_F32 ? static_cast<const float*>(p)[i] : __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ void store_from_float(void* p, int dt, int64_t i, float v) {
  if (dt == ULM_F32)
    static_cast<float*>(p)[i] = v;
  else
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ float round_to(int dt, float v) {
  return dt == ULM_F32 ? v : __bfloat162float(__float2bfloat16_rn(v));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(32 * NORM_WARPS)
    rms_norm_fwd_kernel(const void* __restrict__ x, int xdt, const float* __restrict__ weight, void* __restrict__ y,
                        int ydt, float* __restrict__ rstd, int64_t rows, int D, float eps) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  for (int64_t r = (int64_t)blockIdx.x * NORM_WARPS + (threadIdx.x >> 5); r < rows;
       r += (int64_t)gridDim.x * NORM_WARPS) {
    const int64_t base = r * D;
    float ss = 0.f;
    for (int i = lane; i < D; i += 32) {
      const float v = load_as_float(x, xdt, base + i);
      ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / (float)D + eps);
    for (int i = lane; i < D; i += 32) {
      const float xh = round_to(xdt, load_as_float(x, xdt, base + i) * rs);
      store_from_float(y, ydt, base + i, xh * weight[i]);
    }
    if (lane == 0 && rstd) rstd[r] = rs;
  }
}

// dx (fp32, plus dx_add when given) and one dweight partial row per CTA (part[blockIdx.x][D]); the CTA's warps take rows
// blockIdx.x * NORM_WARPS + warp, then every gridDim.x * NORM_WARPS rows, and keep their column sums
// in shared memory (D floats per warp), added in warp order at the end.
__global__ void __launch_bounds__(32 * NORM_WARPS)
    rms_norm_bwd_kernel(const void* __restrict__ dy, int dydt, const void* __restrict__ x, int xdt,
                        const float* __restrict__ weight, const float* __restrict__ rstd, float* __restrict__ dx,
                        const float* __restrict__ dx_add, float* __restrict__ part, int64_t rows, int D) {
  pdl_enter();
  extern __shared__ float colsum[];  // NORM_WARPS x D
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* mine = colsum + (int64_t)warp * D;
  for (int i = lane; i < D; i += 32) mine[i] = 0.f;
  for (int64_t r = (int64_t)blockIdx.x * NORM_WARPS + warp; r < rows; r += (int64_t)gridDim.x * NORM_WARPS) {
    const int64_t base = r * D;
    const float rs = rstd[r];
    float dot = 0.f;
    for (int i = lane; i < D; i += 32) {
      const float g = load_as_float(dy, dydt, base + i);
      const float xh = load_as_float(x, xdt, base + i) * rs;
      dot = fmaf(g * weight[i], xh, dot);
      mine[i] = fmaf(g, round_to(xdt, xh), mine[i]);
    }
    dot = warp_sum(dot) / (float)D;
    for (int i = lane; i < D; i += 32) {
      const float g = load_as_float(dy, dydt, base + i);
      const float xh = load_as_float(x, xdt, base + i) * rs;
      const float d = rs * (g * weight[i] - xh * dot);
      dx[base + i] = dx_add ? d + dx_add[base + i] : d;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float s = 0.f;
    for (int w = 0; w < NORM_WARPS; ++w) s += colsum[(int64_t)w * D + i];
    part[(int64_t)blockIdx.x * D + i] = s;
  }
}

// The same two kernels for fp32 rows with D % 4 == 0 and D <= 128 * NV: each lane keeps its
// float4 columns (lane, lane + 32, ...) of the row in registers, so the row is read once per pass.
template <int NV>
__global__ void __launch_bounds__(32 * NORM_WARPS)
    rms_norm_fwd_vec_kernel(const float* __restrict__ x, const float* __restrict__ weight, float* __restrict__ y,
                            float* __restrict__ rstd, int64_t rows, int D, float eps) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int D4 = D / 4;
  for (int64_t r = (int64_t)blockIdx.x * NORM_WARPS + (threadIdx.x >> 5); r < rows;
       r += (int64_t)gridDim.x * NORM_WARPS) {
    const float4* xr = reinterpret_cast<const float4*>(x + r * D);
    float4 v[NV];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = lane + 32 * j;
      v[j] = i < D4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      ss = fmaf(v[j].x, v[j].x, fmaf(v[j].y, v[j].y, fmaf(v[j].z, v[j].z, fmaf(v[j].w, v[j].w, ss))));
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / (float)D + eps);
    float4* yr = reinterpret_cast<float4*>(y + r * D);
    const float4* w4 = reinterpret_cast<const float4*>(weight);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = lane + 32 * j;
      if (i < D4) {
        const float4 w = w4[i];
        yr[i] = make_float4(v[j].x * rs * w.x, v[j].y * rs * w.y, v[j].z * rs * w.z, v[j].w * rs * w.w);
      }
    }
    if (lane == 0 && rstd) rstd[r] = rs;
  }
}

template <int NV>
__global__ void __launch_bounds__(32 * NORM_WARPS, NV <= 6 ? 2 : 1)  // two CTAs per SM up to NV = 6
    rms_norm_bwd_vec_kernel(const float* __restrict__ dy, const float* __restrict__ x, const float* __restrict__ weight,
                            const float* __restrict__ rstd, float* __restrict__ dx,
                            const float* __restrict__ dx_add, float* __restrict__ part, int64_t rows, int D) {
  pdl_enter();
  extern __shared__ float colsum[];  // NORM_WARPS x D
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int D4 = D / 4;
  float4* mine = reinterpret_cast<float4*>(colsum + (int64_t)warp * D);
  const float4* w4 = reinterpret_cast<const float4*>(weight);
  float4 acc[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t r = (int64_t)blockIdx.x * NORM_WARPS + warp; r < rows; r += (int64_t)gridDim.x * NORM_WARPS) {
    const float rs = rstd[r];
    const float4* gr = reinterpret_cast<const float4*>(dy + r * D);
    const float4* xr = reinterpret_cast<const float4*>(x + r * D);
    float4 g[NV], xh[NV], ad[NV];
    const float4* ar = dx_add ? reinterpret_cast<const float4*>(dx_add + r * D) : nullptr;
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = lane + 32 * j;
      g[j] = i < D4 ? gr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      ad[j] = (dx_add && i < D4) ? ar[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 xv = i < D4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      xh[j] = make_float4(xv.x * rs, xv.y * rs, xv.z * rs, xv.w * rs);
      const float4 w = i < D4 ? w4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      dot = fmaf(g[j].x * w.x, xh[j].x, fmaf(g[j].y * w.y, xh[j].y,
                 fmaf(g[j].z * w.z, xh[j].z, fmaf(g[j].w * w.w, xh[j].w, dot))));
      acc[j].x = fmaf(g[j].x, xh[j].x, acc[j].x);
      acc[j].y = fmaf(g[j].y, xh[j].y, acc[j].y);
      acc[j].z = fmaf(g[j].z, xh[j].z, acc[j].z);
      acc[j].w = fmaf(g[j].w, xh[j].w, acc[j].w);
    }
    dot = warp_sum(dot) / (float)D;
    float4* dr = reinterpret_cast<float4*>(dx + r * D);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = lane + 32 * j;
      if (i < D4) {
        const float4 w = w4[i];
        float4 d = make_float4(rs * (g[j].x * w.x - xh[j].x * dot), rs * (g[j].y * w.y - xh[j].y * dot),
                               rs * (g[j].z * w.z - xh[j].z * dot), rs * (g[j].w * w.w - xh[j].w * dot));
        if (dx_add) d = make_float4(d.x + ad[j].x, d.y + ad[j].y, d.z + ad[j].z, d.w + ad[j].w);
        dr[i] = d;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = lane + 32 * j;
    if (i < D4) mine[i] = acc[j];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float t = 0.f;
    for (int w = 0; w < NORM_WARPS; ++w) t += colsum[(int64_t)w * D + i];
    part[(int64_t)blockIdx.x * D + i] = t;
  }
}

// CTAs of the RMSNorm kernels: enough rows in flight, at most four CTAs per SM (each writes one
// partial dweight row in the backward)
int norm_grid(int64_t rows) {
  const int dev = current_device();
  const int64_t cap = 4LL * (dev >= 0 ? sm_count(dev) : 148);
  return (int)std::max<int64_t>(1, std::min<int64_t>(cap, cdiv(rows, NORM_WARPS)));
}

}  // namespace
}  // namespace ulm

using namespace ulm;

extern "C" int ulm_rms_norm_fwd(const void* x, int x_dtype, const float* weight, void* y, int y_dtype, float* rstd,
                                int64_t rows, int64_t D, float eps, void* stream) {
  ULM_REQUIRE(rows >= 0 && D >= 0, "negative extent");
  ULM_REQUIRE((x_dtype == ULM_F32 || x_dtype == ULM_BF16) && (y_dtype == ULM_F32 || y_dtype == ULM_BF16),
              "x_dtype and y_dtype must be ULM_F32 or ULM_BF16");
  ULM_REQUIRE(D < (1 << 30), "extent too large");
  if (rows == 0 || D == 0) return ULM_OK;
  ULM_REQUIRE(x && weight && y, "null pointer argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)norm_grid(rows)), block(32 * NORM_WARPS);
  if (x_dtype == ULM_F32 && y_dtype == ULM_F32 && D % 4 == 0 && is_aligned16(x) && is_aligned16(y) &&
      is_aligned16(weight)) {
    const float* xf = static_cast<const float*>(x);
    float* yf = static_cast<float*>(y);
    if (D <= 128 * 4)
      return launch_pdl(rms_norm_fwd_vec_kernel<4>, grid, block, 0, st, xf, weight, yf, rstd, rows, (int)D, eps);
    if (D <= 128 * 8)
      return launch_pdl(rms_norm_fwd_vec_kernel<8>, grid, block, 0, st, xf, weight, yf, rstd, rows, (int)D, eps);
  }
  return launch_pdl(rms_norm_fwd_kernel, grid, block, 0, st, x, x_dtype, weight, y, y_dtype, rstd, rows, (int)D, eps);
}

extern "C" int64_t ulm_rms_norm_bwd_work_bytes(int64_t rows, int64_t D) {
  if (rows < 0 || D < 0) return -1;
  return (int64_t)norm_grid(rows) * D * (int64_t)sizeof(float);
}

extern "C" int ulm_rms_norm_bwd(const void* dy, int dy_dtype, const void* x, int x_dtype, const float* weight,
                                const float* rstd, float* dx, const float* dx_add, float* dweight, void* work,
                                int64_t rows, int64_t D, void* stream) {
  ULM_REQUIRE(rows >= 0 && D >= 0, "negative extent");
  ULM_REQUIRE((x_dtype == ULM_F32 || x_dtype == ULM_BF16) && (dy_dtype == ULM_F32 || dy_dtype == ULM_BF16),
              "x_dtype and dy_dtype must be ULM_F32 or ULM_BF16");
  ULM_REQUIRE(D < (1 << 30) && D * NORM_WARPS * (int64_t)sizeof(float) <= 200 * 1024,
              "rows longer than the backward's shared-memory column sums allow");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (D == 0) return ULM_OK;
  ULM_REQUIRE(dweight, "null pointer argument");
  if (rows == 0) {
    ULM_CUDA_TRY(cudaMemsetAsync(dweight, 0, D * sizeof(float), st));
    return ULM_OK;
  }
  ULM_REQUIRE(dy && x && weight && rstd && dx && work, "null pointer argument");
  const int grid = norm_grid(rows);
  const size_t smem = (size_t)NORM_WARPS * D * sizeof(float);
  if (smem > 48 * 1024)
    ULM_CUDA_TRY(cudaFuncSetAttribute(rms_norm_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  float* part = static_cast<float*>(work);
  const bool vec = x_dtype == ULM_F32 && dy_dtype == ULM_F32 && D % 4 == 0 && D <= 128 * 8 && is_aligned16(x) &&
                   is_aligned16(dy) && is_aligned16(dx) && is_aligned16(weight) && (!dx_add || is_aligned16(dx_add));
  if (vec) {
    const float* xf = static_cast<const float*>(x);
    const float* gf = static_cast<const float*>(dy);
    // float4s per lane: the row's D / 4 over 32 lanes, rounded up to an even count (registers)
    const int64_t nv = cdiv(D / 4, 32);
    auto kern = nv <= 2   ? rms_norm_bwd_vec_kernel<2>
                : nv <= 4 ? rms_norm_bwd_vec_kernel<4>
                : nv <= 6 ? rms_norm_bwd_vec_kernel<6>
                          : rms_norm_bwd_vec_kernel<8>;
    if (smem > 48 * 1024)
      ULM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    if (int rc = launch_pdl(kern, dim3((unsigned)grid), dim3(32 * NORM_WARPS), smem, st, gf, xf, weight, rstd, dx,
                            dx_add, part, rows, (int)D))
      return rc;
  } else if (int rc = launch_pdl(rms_norm_bwd_kernel, dim3((unsigned)grid), dim3(32 * NORM_WARPS), smem, st, dy,
                                 dy_dtype, x, x_dtype, weight, rstd, dx, dx_add, part, rows, (int)D)) {
    return rc;
  }
  // dweight = the CTAs' partial rows summed in a fixed order (a tree over the parts: there are many)
  return sum_parts(static_cast<const float*>(part), grid, D, dweight, st);
}

// ---- Linear -------------------------------------------------------------------------------------

extern "C" int ulm_linear_fwd(const void* x, int x_dtype, const float* weight, void* x_op, void* w_op, void* y,
                              int y_dtype, int64_t N, int64_t K, int64_t Nout, int prec, void* stream) {
  ULM_REQUIRE(prec == ULM_PREC_BF16 || prec == ULM_PREC_FP32, "prec must be ULM_PREC_BF16 or ULM_PREC_FP32");
  ULM_REQUIRE((x_dtype == ULM_F32 || x_dtype == ULM_BF16) && (y_dtype == ULM_F32 || y_dtype == ULM_BF16),
              "x_dtype and y_dtype must be ULM_F32 or ULM_BF16");
  ULM_REQUIRE(N >= 0 && K >= 0 && Nout >= 0, "negative extent");
  ULM_REQUIRE(N < (1ll << 31) && K < (1 << 30) && Nout < (1 << 30), "extent too large");
  if (N == 0 || Nout == 0) return ULM_OK;
  ULM_REQUIRE(x && weight && x_op && w_op && y, "null pointer argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K == 0) {
    ULM_CUDA_TRY(cudaMemsetAsync(y, 0, N * Nout * (y_dtype == ULM_F32 ? 4 : 2), st));
    return ULM_OK;
  }
  const int dt = op_dtype_of(prec);
  const int64_t ldk = ulm_operand_ld(K);
  if (int rc = convert_rows(x, x_dtype, K, x_op, dt, ldk, N, K, st)) return rc;
  if (int rc = convert_rows(weight, ULM_F32, K, w_op, dt, ldk, Nout, K, st)) return rc;
  // y[n][o] = sum_k x[n][k] W[o][k]: both operands K-major, one "batch"
  Operand A{x_op, ldk, N * ldk, K, N, dt, false};
  Operand Bw{w_op, ldk, Nout * ldk, K, Nout, dt, false};
  GemmShape s{1, (int)N, (int)Nout, (int)K, CAUSAL_NONE};
  GemmEpilogue e = make_epilogue(EPI_STORE, y_dtype, y, Nout, 0, nullptr);
  return run_gemm(A, Bw, s, e, st);
}

extern "C" int64_t ulm_linear_bwd_work_bytes(int64_t N, int64_t K, int64_t Nout, int prec) {
  if (N < 0 || K < 0 || Nout < 0 || (prec != ULM_PREC_BF16 && prec != ULM_PREC_FP32)) return -1;
  const int64_t es = prec == ULM_PREC_FP32 ? 4 : 2;
  // dy's operand copy, then the split-K partials of dW (at most 8)
  return align256(N * ulm_operand_ld(Nout) * es) + 8 * Nout * K * (int64_t)sizeof(float);
}

extern "C" int ulm_linear_bwd(const void* dy, int dy_dtype, const void* x_op, const void* w_op, float* dx,
                              const float* dx_add, float* dw, void* work, int64_t N, int64_t K, int64_t Nout, int prec,
                              void* stream) {
  ULM_REQUIRE(prec == ULM_PREC_BF16 || prec == ULM_PREC_FP32, "prec must be ULM_PREC_BF16 or ULM_PREC_FP32");
  ULM_REQUIRE(dy_dtype == ULM_F32 || dy_dtype == ULM_BF16, "dy_dtype must be ULM_F32 or ULM_BF16");
  ULM_REQUIRE(N >= 0 && K >= 0 && Nout >= 0, "negative extent");
  ULM_REQUIRE(N < (1ll << 31) && K < (1 << 30) && Nout < (1 << 30), "extent too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K == 0) return ULM_OK;
  ULM_REQUIRE(dx && dw, "null pointer argument");
  if (N == 0 || Nout == 0) {
    if (N > 0 && dx_add)
      ULM_CUDA_TRY(cudaMemcpyAsync(dx, dx_add, N * K * sizeof(float), cudaMemcpyDeviceToDevice, st));
    else if (N > 0)
      ULM_CUDA_TRY(cudaMemsetAsync(dx, 0, N * K * sizeof(float), st));
    if (Nout > 0) ULM_CUDA_TRY(cudaMemsetAsync(dw, 0, Nout * K * sizeof(float), st));
    return ULM_OK;
  }
  ULM_REQUIRE(dy && x_op && w_op && work, "null pointer argument");
  const int dt = op_dtype_of(prec);
  const int64_t ldk = ulm_operand_ld(K), ldo = ulm_operand_ld(Nout);
  float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(work) + align256(N * ldo * (dt == ULM_F32 ? 4 : 2)));
  // dy is its own operand when it already has the operand type, an unpadded row stride and an
  // aligned start (a bf16 activation gradient); otherwise it is copied into the work buffer
  const void* dy_op = dy;
  if (dy_dtype != dt || ldo != Nout || !is_aligned16(dy)) {
    if (int rc = convert_rows(dy, dy_dtype, Nout, work, dt, ldo, N, Nout, st)) return rc;
    dy_op = work;
  }
  {
    // dx[n][k] = sum_o dy[n][o] W[o][k]: W read as [o][k] = MN-major over k
    Operand A{dy_op, ldo, N * ldo, Nout, N, dt, false};
    Operand Bw{w_op, ldk, Nout * ldk, K, Nout, dt, true};
    GemmShape s{1, (int)N, (int)K, (int)Nout, CAUSAL_NONE};
    GemmEpilogue e = make_epilogue(dx_add ? EPI_STORE_ADD : EPI_STORE, ULM_F32, dx, K, 0, nullptr);
    if (dx_add) {  // dx = dy W + dx_add in the product's epilogue
      e.aux = dx_add;
      e.ld_aux = K;
      e.aux_bstride = 0;
      e.vec_ok = e.vec_ok && is_aligned16(dx_add);
    }
    if (int rc = run_gemm(A, Bw, s, e, st)) return rc;
  }
  // dW[o][k] = sum_n dy[n][o] x[n][k], split K over the rows so the few output tiles fill the GPU
  const int S = fill_split(N, Nout, K);
  Operand A{dy_op, ldo, 0, Nout, N, dt, true};
  Operand Bx{x_op, ldk, 0, K, N, dt, true};
  GemmShape s{S, (int)Nout, (int)K, (int)N, CAUSAL_NONE};
  s.ksplit = S;
  GemmEpilogue e = make_epilogue(EPI_STORE, ULM_F32, S > 1 ? part : dw, K, Nout * K, nullptr);
  if (int rc = run_gemm(A, Bx, s, e, st)) return rc;
  if (S > 1) return sum_parts(static_cast<const float*>(part), S, Nout * K, dw, st);
  return ULM_OK;
}
