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
#include <cstring>

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

template <typename InT>
__device__ __forceinline__ float4 ld4(const void* p, int64_t i);
template <>
__device__ __forceinline__ float4 ld4<float>(const void* p, int64_t i) {
  return *reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
}
template <>
__device__ __forceinline__ float4 ld4<__nv_bfloat16>(const void* p, int64_t i) {
  const uint2 raw = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p) + i);
  __nv_bfloat162 a, b;
  memcpy(&a, &raw.x, 4);
  memcpy(&b, &raw.y, 4);
  const float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

__device__ __forceinline__ void st4(void* p, int64_t i, float4 v, int dt) {
  if (dt == ULM_F32) {
    *reinterpret_cast<float4*>(static_cast<float*>(p) + i) = v;
  } else {
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
    uint2 raw;
    memcpy(&raw.x, &a, 4);
    memcpy(&raw.y, &b, 4);
    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p) + i) = raw;
  }
}

__device__ __forceinline__ float4 fma4(float4 w, float4 x, float4 acc) {
  return make_float4(fmaf(w.x, x.x, acc.x), fmaf(w.y, x.y, acc.y), fmaf(w.z, x.z, acc.z), fmaf(w.w, x.w, acc.w));
}

constexpr int CONV_ROWS = 32;    // positions per CTA of the conv kernels
constexpr int CONV_UNROLL = 4;   // positions per step of a thread's sliding window (loads in flight)
constexpr int CONV_MAXK = 8;

// u[b,t,d] = sum_j conv_w[d, j] * h[b, t-K+1+j, d] (zero before the sequence start).
// CTA = (batch row, CONV_ROWS positions); a thread owns 4 channels and slides a window of the last
// K rows of h down its positions, so every row of h is read once (plus K-1 halo rows).
template <typename InT, int K>
__global__ void __launch_bounds__(256)
    addr_conv_kernel(const void* __restrict__ h, const float* __restrict__ conv_w, void* __restrict__ u, int u_dtype,
                     int64_t ld_u, int T, int D) {
  pdl_enter();
  const int b = blockIdx.y;
  const int t0 = blockIdx.x * CONV_ROWS, t1 = min(T, t0 + CONV_ROWS);
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int d4 = threadIdx.x * 4; d4 < D; d4 += blockDim.x * 4) {
    float4 w[K];
#pragma unroll
    for (int j = 0; j < K; ++j)
      w[j] = make_float4(conv_w[(d4 + 0) * K + j], conv_w[(d4 + 1) * K + j], conv_w[(d4 + 2) * K + j],
                         conv_w[(d4 + 3) * K + j]);
    float4 win[K - 1 + CONV_UNROLL];  // win[j] = h[t - K + 1 + j] for the CONV_UNROLL positions from t
#pragma unroll
    for (int j = 0; j < K - 1; ++j) {
      const int tt = t0 - K + 1 + j;
      win[j] = tt >= 0 ? ld4<InT>(h, ((int64_t)b * T + tt) * D + d4) : z4;
    }
    for (int t = t0; t < t1; t += CONV_UNROLL) {
#pragma unroll
      for (int i = 0; i < CONV_UNROLL; ++i)  // all loads of the step first
        win[K - 1 + i] = t + i < t1 ? ld4<InT>(h, ((int64_t)b * T + t + i) * D + d4) : z4;
#pragma unroll
      for (int i = 0; i < CONV_UNROLL; ++i) {
        if (t + i < t1) {
          float4 acc = z4;
#pragma unroll
          for (int j = 0; j < K; ++j) acc = fma4(w[j], win[i + j], acc);
          st4(u, ((int64_t)b * T + t + i) * ld_u + d4, acc, u_dtype);
        }
      }
#pragma unroll
      for (int j = 0; j < K - 1; ++j) win[j] = win[CONV_UNROLL + j];
    }
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

// den[row] = eps + sum of the row's partial sums, written by the key GEMM's epilogue (one per
// column block, unused slots zero), summed in a fixed order
__global__ void addr_den_kernel(const float* __restrict__ part, int part_ld, const float* __restrict__ eps,
                                float* __restrict__ den, int64_t rows) {
  pdl_enter();
  const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const float* p = part + row * part_ld;
  float s = 0.f;
  for (int j = 0; j < part_ld; ++j) s += p[j];
  den[row] = *eps + s;
}

// one warp per row: s = sum dr r, then da = 2 sqrt(r den) (dr - s) / den; -s/den summed per CTA
// (d eps partial). With `unnormalised`, x holds z = r den instead of r: s = sum dr z / den and
// da = 2 sqrt(z) (dr - s) / den. Rows are read with 16-byte loads; the second pass over a row hits L1.
__global__ void __launch_bounds__(256)
    addr_bwd_kernel(const float* __restrict__ dr, const float* __restrict__ r, const float* __restrict__ den,
                    int unnormalised, void* __restrict__ da, int da_dtype, int64_t ld_da,
                    float* __restrict__ deps_part, int64_t rows, int M, int rows_per_cta) {
  pdl_enter();
  __shared__ float deps_w[8];
  const int wp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float deps_acc = 0.f;
  const int64_t row0 = (int64_t)blockIdx.x * rows_per_cta;
  for (int rr = wp; rr < rows_per_cta; rr += 8) {
    const int64_t row = row0 + rr;
    if (row >= rows) break;
    const float* drr = dr + row * M;
    const float* rrow = r + row * M;
    const float dn = den[row];  // issued first: its latency hides behind the row's loads
    float s = 0.f;
    int m = lane * 4;
    // four 16-byte loads of each array in flight, then the products in the same order as one by one
    for (; m + 384 < M; m += 512) {
      float4 a[4], c[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        a[u] = *reinterpret_cast<const float4*>(drr + m + 128 * u);
        c[u] = *reinterpret_cast<const float4*>(rrow + m + 128 * u);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        s = fmaf(a[u].x, c[u].x, fmaf(a[u].y, c[u].y, fmaf(a[u].z, c[u].z, fmaf(a[u].w, c[u].w, s))));
    }
    for (; m < M; m += 128) {
      const float4 a = *reinterpret_cast<const float4*>(drr + m);
      const float4 c = *reinterpret_cast<const float4*>(rrow + m);
      s = fmaf(a.x, c.x, fmaf(a.y, c.y, fmaf(a.z, c.z, fmaf(a.w, c.w, s))));
    }
    s = warp_sum(s);
    const float inv = 1.0f / dn;
    // z scale: sqrt(z) = sqrt(x * zs) with zs = den for normalised rows, 1 for z rows
    const float zs = unnormalised ? 1.f : dn;
    if (unnormalised) s *= inv;
    deps_acc -= s * inv;
    // second pass over the row (mostly cache hits), four loads of each array in flight as well
    m = lane * 4;
    for (; m + 384 < M; m += 512) {
      float4 a4[4], c4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        a4[u] = *reinterpret_cast<const float4*>(drr + m + 128 * u);
        c4[u] = *reinterpret_cast<const float4*>(rrow + m + 128 * u);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4 a = a4[u], c = c4[u];
        float4 o;
        o.x = 2.f * sqrtf(c.x * zs) * ((a.x - s) * inv);
        o.y = 2.f * sqrtf(c.y * zs) * ((a.y - s) * inv);
        o.z = 2.f * sqrtf(c.z * zs) * ((a.z - s) * inv);
        o.w = 2.f * sqrtf(c.w * zs) * ((a.w - s) * inv);
        st4(da, row * ld_da + m + 128 * u, o, da_dtype);
      }
    }
    for (; m < M; m += 128) {
      const float4 a = *reinterpret_cast<const float4*>(drr + m);
      const float4 c = *reinterpret_cast<const float4*>(rrow + m);
      float4 o;
      o.x = 2.f * sqrtf(c.x * zs) * ((a.x - s) * inv);
      o.y = 2.f * sqrtf(c.y * zs) * ((a.y - s) * inv);
      o.z = 2.f * sqrtf(c.z * zs) * ((a.z - s) * inv);
      o.w = 2.f * sqrtf(c.w * zs) * ((a.w - s) * inv);
      st4(da, row * ld_da + m, o, da_dtype);
    }
  }
  if (lane == 0) deps_w[wp] = deps_acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += deps_w[w];
    deps_part[blockIdx.x] = t;
  }
}

// The address backward with each row held in registers: a CTA's 8 warps form two row groups of
// four warps, each warp holding a quarter of the row (NV4 16-byte loads per lane and array), so a
// row is read from HBM once, all its loads in flight together, and da is computed from the
// registers. The quarter sums meet in shared memory (a named barrier per group) and are added in
// quarter order (each warp's sum is formed from NV4 independent partial sums); da per element is
// addr_bwd_kernel's arithmetic. Needs M % 16 == 0 and M / 4 <= 128 * NV4; FULL: M / 4 == 128 * NV4.
// named barrier of one four-warp row group (ids 1 and 2; literal ids keep the CTA at three barriers)
__device__ __forceinline__ void group_bar(int grp) {
  if (grp == 0)
    asm volatile("bar.sync 1, 128;" ::: "memory");
  else
    asm volatile("bar.sync 2, 128;" ::: "memory");
}

template <int NV4, bool FULL>
__global__ void __launch_bounds__(256)
    addr_bwd_rows_kernel(const float* __restrict__ dr, const float* __restrict__ r, const float* __restrict__ den,
                         int unnormalised, void* __restrict__ da, int da_dtype, int64_t ld_da,
                         float* __restrict__ deps_part, int64_t rows, int M, int rows_per_cta) {
  pdl_enter();
  __shared__ float qsum[2][4];
  __shared__ float deps_g[2];
  const int wp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = wp >> 2, qt = wp & 3;  // row group, quarter of the row
  const int Mq = M >> 2;
  float deps_acc = 0.f;
  const int64_t row0 = (int64_t)blockIdx.x * rows_per_cta;
  for (int rr = grp; rr < rows_per_cta; rr += 2) {
    const int64_t row = row0 + rr;
    if (row >= rows) break;  // the group's four warps leave together
    const float* drr = dr + row * M + qt * Mq;
    const float* rrow = r + row * M + qt * Mq;
    const float dn = den[row];
    float4 a[NV4], c[NV4];
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
      const int m = (i * 32 + lane) * 4;
      if (FULL || m < Mq) {
        a[i] = *reinterpret_cast<const float4*>(drr + m);
        c[i] = *reinterpret_cast<const float4*>(rrow + m);
      } else {
        a[i] = c[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    // one partial sum per 16-byte load (independent chains), added in load order
    float sp[NV4];
#pragma unroll
    for (int i = 0; i < NV4; ++i) sp[i] = fmaf(a[i].x, c[i].x, fmaf(a[i].y, c[i].y, fmaf(a[i].z, c[i].z, a[i].w * c[i].w)));
    float s = sp[0];
#pragma unroll
    for (int i = 1; i < NV4; ++i) s += sp[i];
    s = warp_sum(s);
    if (lane == 0) qsum[grp][qt] = s;
    group_bar(grp);
    s = ((qsum[grp][0] + qsum[grp][1]) + qsum[grp][2]) + qsum[grp][3];
    group_bar(grp);  // qsum is free for the group's next row
    const float inv = 1.0f / dn;
    // z scale: sqrt(z) = sqrt(x * zs) with zs = den for normalised rows, 1 for z rows
    const float zs = unnormalised ? 1.f : dn;
    if (unnormalised) s *= inv;
    deps_acc -= s * inv;
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
      const int m = (i * 32 + lane) * 4;
      if (FULL || m < Mq) {
        float4 o;
        o.x = 2.f * sqrtf(c[i].x * zs) * ((a[i].x - s) * inv);
        o.y = 2.f * sqrtf(c[i].y * zs) * ((a[i].y - s) * inv);
        o.z = 2.f * sqrtf(c[i].z * zs) * ((a[i].z - s) * inv);
        o.w = 2.f * sqrtf(c[i].w * zs) * ((a[i].w - s) * inv);
        st4(da, row * ld_da + qt * Mq + m, o, da_dtype);
      }
    }
  }
  if (qt == 0 && lane == 0) deps_g[grp] = deps_acc;
  __syncthreads();
  if (threadIdx.x == 0) deps_part[blockIdx.x] = deps_g[0] + deps_g[1];
}

// column sums of a bf16 (rows x cols) array over chunks of rows, part[chunk][col]: a CTA covers
// 256 columns (8 per lane, one 16-byte load per row: a warp reads 512 contiguous bytes) of one chunk;
// warp w adds rows w, w + 8, ... of the chunk in order, then the warps' sums are added in warp order.
__global__ void __launch_bounds__(256)
    col_sum_bf16x8_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld, int64_t rows, int cols,
                          int rows_per_chunk, float* __restrict__ part) {
  pdl_enter();
  __shared__ float red[8][257];
  const int wp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = blockIdx.x * 256 + lane * 8;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_chunk;
  const int64_t r1 = min(rows, r0 + rows_per_chunk);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (c0 < cols) {
#pragma unroll 4
    for (int64_t rr = r0 + wp; rr < r1; rr += 8) {
      const uint4 pk = *reinterpret_cast<const uint4*>(x + rr * ld + c0);
      const uint32_t w4[4] = {pk.x, pk.y, pk.z, pk.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 h;
        memcpy(&h, &w4[j], 4);
        const float2 f = __bfloat1622float2(h);
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[wp][lane * 8 + j] = acc[j];
  __syncthreads();
  const int col = blockIdx.x * 256 + threadIdx.x;
  if (col < cols) {
    float t = red[0][threadIdx.x];
#pragma unroll
    for (int w = 1; w < 8; ++w) t += red[w][threadIdx.x];
    part[(int64_t)blockIdx.y * cols + col] = t;
  }
}

// column sums of a (rows x cols) operand-type array over chunks of rows: part[chunk][col]
template <typename InT>
__global__ void col_sum_kernel(const void* __restrict__ x, int64_t ld, int64_t rows, int cols, int rows_per_chunk,
                               float* __restrict__ part) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= cols) return;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_chunk;
  const int64_t r1 = min(rows, r0 + rows_per_chunk);
  float s = 0.f;
  for (int64_t rr = r0; rr < r1; ++rr) s += ld_as_float<InT>(x, rr * ld + col);
  part[(int64_t)blockIdx.y * cols + col] = s;
}

// out[g][i] = sum of part[p][i] over the parts p of group g (parts g * per .. g * per + per - 1, in
// order): one thread per 4 consecutive outputs, blockIdx.y = group; n % 4 == 0, 16-byte aligned rows
__global__ void __launch_bounds__(256)
    sum_groups4_kernel(const float* __restrict__ part, int64_t nparts, int64_t n, int64_t per, float* __restrict__ out) {
  pdl_enter();
  const int64_t i = ((int64_t)blockIdx.x * 256 + threadIdx.x) * 4;
  if (i >= n) return;
  const int64_t p0 = (int64_t)blockIdx.y * per, p1 = min(nparts, p0 + per);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
  for (int64_t p = p0; p < p1; ++p) {
    const float4 a = *reinterpret_cast<const float4*>(part + p * n + i);
    acc.x += a.x;
    acc.y += a.y;
    acc.z += a.z;
    acc.w += a.w;
  }
  *reinterpret_cast<float4*>(out + (int64_t)blockIdx.y * n + i) = acc;
}

// out[i] = sum over p of part[p][i] for many parts and few outputs: a CTA covers 8 groups of 4
// consecutive outputs; its 32 part lanes (threadIdx.x / 8) add parts lane, lane + 32, ... in order,
// then the 32 lane sums are added by a fixed tree. n % 4 == 0, 16-byte aligned rows.
__global__ void __launch_bounds__(256)
    sum_parts_tree_kernel(const float* __restrict__ part, int64_t nparts, int64_t n, float* __restrict__ out) {
  pdl_enter();
  __shared__ float4 red[32][8];
  const int c = threadIdx.x & 7, pl = threadIdx.x >> 3;
  const int64_t i = ((int64_t)blockIdx.x * 8 + c) * 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (i < n) {
    // parts pl, pl + 32, ... added in that order; eight loads in flight per step
    int64_t p = pl;
    for (; p + 32 * 7 < nparts; p += 32 * 8) {
      float4 a[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) a[u] = *reinterpret_cast<const float4*>(part + (p + 32 * u) * n + i);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        acc.x += a[u].x;
        acc.y += a[u].y;
        acc.z += a[u].z;
        acc.w += a[u].w;
      }
    }
    for (; p < nparts; p += 32) {
      const float4 a = *reinterpret_cast<const float4*>(part + p * n + i);
      acc.x += a.x;
      acc.y += a.y;
      acc.z += a.z;
      acc.w += a.w;
    }
  }
  red[pl][c] = acc;
  __syncthreads();
  for (int st = 16; st > 0; st >>= 1) {
    if (pl < st) {
      const float4 b = red[pl + st][c];
      float4& a = red[pl][c];
      a.x += b.x;
      a.y += b.y;
      a.z += b.z;
      a.w += b.w;
    }
    __syncthreads();
  }
  if (pl == 0 && i < n) *reinterpret_cast<float4*>(out + i) = red[0][c];
}

// out[i] = sum_p part[p][i] over nparts, in order (any n)
__global__ void sum_parts_kernel(const float* __restrict__ part, int64_t nparts, int64_t n, float* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int64_t p = 0; p < nparts; ++p) s += part[p * n + i];
    out[i] = s;
  }
}

// deterministic sum of n floats into *out (one block)
__global__ void __launch_bounds__(256) sum_all_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ out) {
  pdl_enter();
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

// dh[t] = sum_j w[j] du[t+K-1-j] and the conv-weight partials dconv[j] += du[t] h[t-K+1+j], CTA =
// (batch row, CONV_ROWS positions), thread = 4 channels with windows of du (ahead) and h (behind);
// each CTA writes its dconv partial, reduced later in a fixed order.
template <typename InT, int K>
__global__ void __launch_bounds__(256)
    addr_conv_bwd_kernel(const float* __restrict__ du, const void* __restrict__ h, const float* __restrict__ conv_w,
                         float* __restrict__ dh, float* __restrict__ dconv_part, int T, int D) {
  pdl_enter();
  const int b = blockIdx.y;
  const int t0 = blockIdx.x * CONV_ROWS, t1 = min(T, t0 + CONV_ROWS);
  const int64_t part = (int64_t)blockIdx.y * gridDim.x + blockIdx.x;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int d4 = threadIdx.x * 4; d4 < D; d4 += blockDim.x * 4) {
    float4 w[K], acc[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
      w[j] = make_float4(conv_w[(d4 + 0) * K + j], conv_w[(d4 + 1) * K + j], conv_w[(d4 + 2) * K + j],
                         conv_w[(d4 + 3) * K + j]);
      acc[j] = z4;
    }
    // for the CONV_UNROLL positions from t: hw[j] = h[t - K + 1 + j], dw[j] = du[t + j]
    float4 hw[K - 1 + CONV_UNROLL];
    float4 dw[K - 1 + CONV_UNROLL];
#pragma unroll
    for (int j = 0; j < K - 1; ++j) {
      const int tt = t0 - K + 1 + j;
      hw[j] = tt >= 0 ? ld4<InT>(h, ((int64_t)b * T + tt) * D + d4) : z4;
      const int tf = t0 + j;
      dw[j] = tf < T ? *reinterpret_cast<const float4*>(du + ((int64_t)b * T + tf) * D + d4) : z4;
    }
    for (int t = t0; t < t1; t += CONV_UNROLL) {
#pragma unroll
      for (int i = 0; i < CONV_UNROLL; ++i) {  // all loads of the step first
        hw[K - 1 + i] = t + i < t1 ? ld4<InT>(h, ((int64_t)b * T + t + i) * D + d4) : z4;
        const int tf = t + K - 1 + i;
        dw[K - 1 + i] = tf < T ? *reinterpret_cast<const float4*>(du + ((int64_t)b * T + tf) * D + d4) : z4;
      }
#pragma unroll
      for (int i = 0; i < CONV_UNROLL; ++i) {
        if (t + i < t1) {
          float4 g = z4;
#pragma unroll
          for (int j = 0; j < K; ++j) g = fma4(w[j], dw[i + K - 1 - j], g);
          *reinterpret_cast<float4*>(dh + ((int64_t)b * T + t + i) * D + d4) = g;
#pragma unroll
          for (int j = 0; j < K; ++j) acc[j] = fma4(dw[i], hw[i + j], acc[j]);
        }
      }
#pragma unroll
      for (int j = 0; j < K - 1; ++j) {
        hw[j] = hw[CONV_UNROLL + j];
        dw[j] = dw[CONV_UNROLL + j];
      }
    }
#pragma unroll
    for (int j = 0; j < K; ++j) {
      dconv_part[(part * D + d4 + 0) * K + j] = acc[j].x;
      dconv_part[(part * D + d4 + 1) * K + j] = acc[j].y;
      dconv_part[(part * D + d4 + 2) * K + j] = acc[j].z;
      dconv_part[(part * D + d4 + 3) * K + j] = acc[j].w;
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
  e.row_partial = nullptr;
  e.part_ld = 0;
  e.staged = 0;
  const int vec = out_dtype == ULM_F32 ? 4 : 8;
  e.vec_ok = is_aligned16(out) && ldo % vec == 0 && bstride % vec == 0;
  return e;
}

struct AddrBwdWork {
  void* da;         // rows x ld_m, op dtype
  float* du;        // rows x D
  float* dk_part;   // S x M x D
  float* db_part;   // db_chunks x M
  float* deps_part; // ctas
  float* dconv_part;
  int64_t ld_m;
  int S, ctas, chunks, db_chunks;
  int64_t bytes;
};

constexpr int ADDR_ROWS_PER_CTA = 32;
constexpr int DB_ROWS_PER_CHUNK = 256;

inline int64_t al256(int64_t n) { return (n + 255) / 256 * 256; }

// Partial sums over more than SUM_GROUP parts use the 32-lane tree kernel.
constexpr int64_t SUM_GROUP = 16;

// Split of the B*T contraction of dK = da^T u into S k ranges: enough 256 x 256 tiles to fill the
// CTA pairs once (S x tiles <= pairs), at most 8, each range at least 1024 rows and none empty.
inline int addr_split(int64_t rows, int64_t M, int64_t D) {
  const int dev = current_device();
  const int pairs = (dev >= 0 ? sm_count(dev) : 148) / 2;
  const int64_t tiles = cdiv(M, 256) * cdiv(D, 256);
  int S = (int)std::max<int64_t>(1, std::min<int64_t>(8, pairs / std::max<int64_t>(1, tiles)));
  while (S > 1 && (rows / S < 1024 || (int64_t)(S - 1) * ksplit_chunk((int)rows, S) >= rows)) --S;
  return S;
}

inline AddrBwdWork carve_addr_work(void* base, int64_t B, int64_t T, int64_t D, int64_t M, int op_dt) {
  AddrBwdWork w;
  const int64_t rows = B * T;
  w.ld_m = ulm_operand_ld(M);
  w.S = addr_split(rows, M, D);
  w.ctas = (int)cdiv(rows, ADDR_ROWS_PER_CTA);
  w.chunks = (int)cdiv(T, CONV_ROWS);
  w.db_chunks = (int)cdiv(rows, DB_ROWS_PER_CHUNK);
  char* p = static_cast<char*>(base);
  char* p0 = p;
  auto take = [&](int64_t bytes) {
    char* q = p;
    p += al256(bytes);
    return q;
  };
  w.da = take(rows * w.ld_m * (op_dt == ULM_F32 ? 4 : 2));
  w.du = reinterpret_cast<float*>(take(rows * D * 4));
  // sized for the largest split so the byte count does not depend on the device queried
  w.dk_part = reinterpret_cast<float*>(take((int64_t)8 * M * D * 4));
  w.db_part = reinterpret_cast<float*>(take((int64_t)w.db_chunks * M * 4));
  w.deps_part = reinterpret_cast<float*>(take((int64_t)w.ctas * 4));
  w.dconv_part = reinterpret_cast<float*>(take((int64_t)w.chunks * B * D * CONV_MAXK * 4));
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
  ULM_REQUIRE(D % 4 == 0 && M % 4 == 0, "the addressing kernels need D %% 4 == 0 and M %% 4 == 0");
  return ULM_OK;
}

}  // namespace

// out = sum of nparts arrays of n floats, in a fixed order: one thread per 4 outputs adding the parts
// in order when they are few (at most SUM_GROUP), else 32 part lanes per output and a fixed tree.
int sum_parts(const float* part, int64_t nparts, int64_t n, float* out, cudaStream_t st) {
  if (n % 4 == 0 && is_aligned16(part) && is_aligned16(out)) {
    if (nparts > SUM_GROUP)
      return launch_pdl(sum_parts_tree_kernel, dim3((unsigned)cdiv(n / 4, 8)), dim3(256), 0, st, part, nparts, n,
                        out);
    return launch_pdl(sum_groups4_kernel, dim3((unsigned)cdiv(n / 4, 256), 1), dim3(256), 0, st, part, nparts, n,
                      nparts, out);
  }
  sum_parts_kernel<<<(unsigned)std::min<int64_t>(cdiv(n, 256), 16 * 148), 256, 0, st>>>(part, nparts, n, out);
  ULM_LAUNCH_CHECK("sum_parts_kernel");
  return ULM_OK;
}

// column blocks of the key GEMM's row partial sums: the narrowest tile of any GEMM back end is 64
int64_t addr_part_ld(int64_t M) { return cdiv(M, 64); }

extern "C" int64_t ulm_address_fwd_work_bytes(int64_t B, int64_t T, int64_t M) {
  return B * T * addr_part_ld(M) * (int64_t)sizeof(float);
}

extern "C" int ulm_address_fwd(const void* h, int h_dtype, const float* conv_w, int64_t conv_size, const void* key_w,
                               int64_t ld_kw, const float* key_b, const float* eps, float* r, float* den,
                               int normalize, void* work, void* u_op, int64_t ld_u, int64_t B, int64_t T, int64_t D,
                               int64_t M, int prec, void* stream) {
  if (int rc = addr_check(h_dtype, prec, B, T, D, M, conv_size)) return rc;
  ULM_REQUIRE(h && conv_w && key_w && key_b && eps && r && den && u_op, "null pointer argument");
  ULM_REQUIRE(normalize || work, "the unnormalised form needs ulm_address_fwd_work_bytes of work");
  ULM_REQUIRE(ld_u >= D && ld_kw >= D, "row stride shorter than the row");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int dt = prec == ULM_PREC_FP32 ? ULM_F32 : ULM_BF16;
  const int64_t rows = B * T;
  dim3 cgrid((unsigned)cdiv(T, CONV_ROWS), (unsigned)B);
  const int cthreads = (int)std::min<int64_t>(256, cdiv(D, 4));
  int crc = ULM_OK;
#define ULM_CONV(KK)                                                                                             \
  if (conv_size == KK)                                                                                           \
    crc = h_dtype == ULM_F32                                                                                     \
              ? launch_pdl(addr_conv_kernel<float, KK>, cgrid, dim3(cthreads), 0, st, h, conv_w, u_op, dt, ld_u, \
                           (int)T, (int)D)                                                                       \
              : launch_pdl(addr_conv_kernel<__nv_bfloat16, KK>, cgrid, dim3(cthreads), 0, st, h, conv_w, u_op,   \
                           dt, ld_u, (int)T, (int)D);
  ULM_CONV(1) ULM_CONV(2) ULM_CONV(3) ULM_CONV(4) ULM_CONV(5) ULM_CONV(6) ULM_CONV(7) ULM_CONV(8)
#undef ULM_CONV
  if (crc) return crc;
  // z = relu(u K^T + b)^2 written into r
  Operand A{u_op, ld_u, rows * ld_u, D, rows, dt, false};
  Operand Bw{key_w, ld_kw, M * ld_kw, D, M, dt, false};
  GemmShape s{1, (int)rows, (int)M, (int)D, CAUSAL_NONE};
  GemmEpilogue e = plain_epilogue(EPI_RELU2, ULM_F32, r, M, rows * M);
  e.aux = key_b;
  if (normalize) {
    if (int rc = run_gemm(A, Bw, s, e, st)) return rc;
    addr_normalize_kernel<<<(unsigned)cdiv(rows, 8), 256, 0, st>>>(r, den, eps, rows, (int)M);
    ULM_LAUNCH_CHECK("addr_normalize_kernel");
    return ULM_OK;
  }
  // z stays unnormalised: the epilogue leaves one row sum per column block, den sums them
  float* part = static_cast<float*>(work);
  const int64_t pld = addr_part_ld(M);
  ULM_CUDA_TRY(cudaMemsetAsync(part, 0, rows * pld * sizeof(float), st));
  e.row_partial = part;
  e.part_ld = (int)pld;
  if (int rc = run_gemm(A, Bw, s, e, st)) return rc;
  if (int rc = launch_pdl(addr_den_kernel, dim3((unsigned)cdiv(rows, 256)), dim3(256), 0, st, (const float*)part,
                          (int)pld, eps, den, rows))
    return rc;
  return ULM_OK;
}

extern "C" int64_t ulm_address_bwd_work_bytes(int64_t B, int64_t T, int64_t D, int64_t M, int prec) {
  return carve_addr_work(nullptr, B, T, D, M, prec == ULM_PREC_FP32 ? ULM_F32 : ULM_BF16).bytes;
}

extern "C" int ulm_address_bwd(const float* dr, const float* r, const float* den, int normalized, const void* u_op,
                               int64_t ld_u,
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
  // da and the d eps partials, then db = column sums of da
  {
    const int unnorm = normalized ? 0 : 1;
    const dim3 grid((unsigned)wk.ctas);
    int rc;
    // rows in registers when a quarter row fits in 8 16-byte loads per lane
    if (M % 16 == 0 && M <= 4096) {
      const int64_t nv = cdiv(M / 4, 128);
      auto go = [&](auto kern) {
        return launch_pdl(kern, grid, dim3(256), 0, st, dr, r, den, unnorm, wk.da, dt, wk.ld_m, wk.deps_part, rows,
                          (int)M, ADDR_ROWS_PER_CTA);
      };
      const bool full = M % 512 == 0 && (M / 512) == (nv <= 1 ? 1 : nv <= 2 ? 2 : nv <= 4 ? 4 : 8);
      if (nv <= 1) rc = full ? go(addr_bwd_rows_kernel<1, true>) : go(addr_bwd_rows_kernel<1, false>);
      else if (nv <= 2) rc = full ? go(addr_bwd_rows_kernel<2, true>) : go(addr_bwd_rows_kernel<2, false>);
      else if (nv <= 4) rc = full ? go(addr_bwd_rows_kernel<4, true>) : go(addr_bwd_rows_kernel<4, false>);
      else rc = full ? go(addr_bwd_rows_kernel<8, true>) : go(addr_bwd_rows_kernel<8, false>);
    } else {
      rc = launch_pdl(addr_bwd_kernel, grid, dim3(256), 0, st, dr, r, den, unnorm, wk.da, dt, wk.ld_m, wk.deps_part,
                      rows, (int)M, ADDR_ROWS_PER_CTA);
    }
    if (rc) return rc;
  }
  // du = da K and the conv backward stay on the caller's stream (launched first); db, deps and
  // dK = da^T u run beside them on the side stream
  cudaStream_t side = nullptr;
  if (int rc = side_stream(&side)) return rc;
  if (int rc = stream_after(side, st)) return rc;
  {
    Operand A{wk.da, wk.ld_m, rows * wk.ld_m, M, rows, dt, false};
    Operand Bw{key_w, ld_kw, M * ld_kw, D, M, dt, true};
    GemmShape s{1, (int)rows, (int)D, (int)M, CAUSAL_NONE};
    GemmEpilogue e = plain_epilogue(EPI_STORE, ULM_F32, wk.du, D, rows * D);
    if (int rc = run_gemm(A, Bw, s, e, st)) return rc;
  }
  if (dt == ULM_BF16 && M % 8 == 0 && wk.ld_m % 8 == 0) {
    dim3 g2((unsigned)cdiv(M, 256), (unsigned)wk.db_chunks);
    if (int rc = launch_pdl(col_sum_bf16x8_kernel, g2, dim3(256), 0, side, static_cast<const __nv_bfloat16*>(wk.da),
                            wk.ld_m, rows, (int)M, DB_ROWS_PER_CHUNK, wk.db_part))
      return rc;
  } else {
    dim3 g2((unsigned)cdiv(M, 256), (unsigned)wk.db_chunks);
    if (dt == ULM_F32)
      col_sum_kernel<float><<<g2, 256, 0, side>>>(wk.da, wk.ld_m, rows, (int)M, DB_ROWS_PER_CHUNK, wk.db_part);
    else
      col_sum_kernel<__nv_bfloat16><<<g2, 256, 0, side>>>(wk.da, wk.ld_m, rows, (int)M, DB_ROWS_PER_CHUNK, wk.db_part);
    ULM_LAUNCH_CHECK("col_sum_kernel");
  }
  if (int rc = sum_parts(wk.db_part, wk.db_chunks, M, dkey_b, side)) return rc;
  if (int rc = launch_pdl(sum_all_kernel, dim3(1), dim3(256), 0, side, (const float*)wk.deps_part, (int64_t)wk.ctas,
                          deps))
    return rc;
  // dK = da^T u, split over S k ranges of rows (split-K product), then the partials summed in order
  {
    Operand A{wk.da, wk.ld_m, rows * wk.ld_m, M, rows, dt, true};
    Operand Bu{u_op, ld_u, rows * ld_u, D, rows, dt, true};
    GemmShape s{wk.S, (int)M, (int)D, (int)rows, CAUSAL_NONE};
    s.ksplit = wk.S;
    GemmEpilogue e = plain_epilogue(EPI_STORE, ULM_F32, wk.dk_part, D, M * D);
    if (int rc = run_gemm(A, Bu, s, e, side)) return rc;
    if (int rc = sum_parts(wk.dk_part, wk.S, M * D, dkey_w, side)) return rc;
  }
  // through the conv
  dim3 grid((unsigned)wk.chunks, (unsigned)B);
  const int cthreads = (int)std::min<int64_t>(256, cdiv(D, 4));
  int crc = ULM_OK;
#define ULM_CONVB(KK)                                                                                           \
  if (conv_size == KK)                                                                                          \
    crc = h_dtype == ULM_F32 ? launch_pdl(addr_conv_bwd_kernel<float, KK>, grid, dim3(cthreads), 0, st,          \
                                          (const float*)wk.du, h, conv_w, dh, wk.dconv_part, (int)T, (int)D)     \
                             : launch_pdl(addr_conv_bwd_kernel<__nv_bfloat16, KK>, grid, dim3(cthreads), 0, st,  \
                                          (const float*)wk.du, h, conv_w, dh, wk.dconv_part, (int)T, (int)D);
  ULM_CONVB(1) ULM_CONVB(2) ULM_CONVB(3) ULM_CONVB(4) ULM_CONVB(5) ULM_CONVB(6) ULM_CONVB(7) ULM_CONVB(8)
#undef ULM_CONVB
  if (crc) return crc;
  if (int rc = sum_parts(wk.dconv_part, (int64_t)wk.chunks * B, D * conv_size, dconv_w, st)) return rc;
  return stream_after(st, side);  // join
}

// The path's whole backward for one block with unnormalised addresses (z, den): the operator backward
// (ulm_memory_bwd, or its fused-combine form ulm_memory_combine_bwd) followed by the prologue
// backward (ulm_address_bwd), as one call so that the statistics' dw / dg reductions run on the
// library's side stream beside the address backward; everything is joined to `stream` on return.
extern "C" int ulm_addressed_memory_bwd(const float* dq_out, const void* dfast, int do_dtype, const float* z,
                                        const float* den, const float* g, const float* w, const float* q,
                                        const float* c, const void* qop, const void* kop, const void* vop,
                                        const void* P, void* doop, void* dS, float* dqf, float* dk, void* partial,
                                        float* dr, void* dv, float* dg, float* dw, const void* u_op, int64_t ld_u,
                                        const void* h, int h_dtype, const float* conv_w, int64_t conv_size,
                                        const void* key_w, int64_t ld_kw, float* dh, float* dconv_w, float* dkey_w,
                                        float* dkey_b, float* deps, void* work, int64_t B, int64_t T, int64_t M,
                                        int64_t D, int prec, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaStream_t side = nullptr;
  if (int rc = side_stream(&side)) return rc;
  int rc = memory_bwd_impl(dq_out, dfast, do_dtype, z, den, g, w, q, c, qop, kop, vop, P, doop, dS, dqf, dk, partial,
                           dr, dv, dg, dw, B, T, M, D, prec, stream, side);
  if (!rc)
    rc = ulm_address_bwd(dr, z, den, 0, u_op, ld_u, h, h_dtype, conv_w, conv_size, key_w, ld_kw, dh, dconv_w, dkey_w,
                         dkey_b, deps, work, B, T, D, M, prec, stream);
  const int jrc = stream_after(st, side);  // also on failure: nothing of the call is left unjoined
  return rc ? rc : jrc;
}

extern "C" int ulm_mixer_bwd(const void* dy, int dy_dtype, const float* z, const float* den, const float* g,
                             const float* w, const float* mu, const float* q, const float* c, const void* qop,
                             const void* kop, const void* vop, const void* P, void* doop, void* dS, void* mw,
                             float* dqf, float* dk, void* partial, float* gpart, float* dr, void* dv, int dv_dtype,
                             float* dg, float* dw, float* dmu, const void* u_op, int64_t ld_u, const void* h,
                             int h_dtype, const float* conv_w, int64_t conv_size, const void* key_w, int64_t ld_kw,
                             float* dh, float* dconv_w, float* dkey_w, float* dkey_b, float* deps, void* work,
                             int64_t B, int64_t T, int64_t M, int64_t D, int prec, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaStream_t side = nullptr;
  if (int rc = side_stream(&side)) return rc;
  int rc = combine_bwd_impl(dy, dy_dtype, z, den, g, w, mu, q, c, qop, kop, vop, P, doop, dS, mw, dqf, dk, partial,
                            gpart, dr, dv, dv_dtype, dg, dw, dmu, B, T, M, D, prec, stream, side);
  if (!rc)
    rc = ulm_address_bwd(dr, z, den, 0, u_op, ld_u, h, h_dtype, conv_w, conv_size, key_w, ld_kw, dh, dconv_w, dkey_w,
                         dkey_b, deps, work, B, T, D, M, prec, stream);
  const int jrc = stream_after(st, side);
  return rc ? rc : jrc;
}
