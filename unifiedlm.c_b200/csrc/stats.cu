// Slot statistics of the fast memory: the decayed running mass n_t of every slot and the posterior
// rescale q = r / (w + n) (forward), and their reverse-time backward.
//
// Both passes are HBM-bound scans along time. A CTA owns 32 consecutive slots of one batch row
// (lane = slot, so every load/store of a warp is one contiguous 128-byte row segment) and splits
// time into 8 segments, one warp each. Pass 1 scans each segment from a zero carry and publishes
// the segment's end value; the carries are combined in shared memory (lam^len per segment); pass 2
// rescans with the true carry and writes the outputs. The second read of r hits L2 (a CTA's slice
// is at most 32 x T x 4 bytes).
#include <cooperative_groups.h>

#include <mutex>

#include "gemm.cuh"

// fixed-order sums of partial arrays (address.cu)
int sum_parts(const float* part, int64_t nparts, int64_t n, float* out, cudaStream_t st);

namespace ulm {

constexpr int STATS_SEGS = 8;
constexpr int STATS_THREADS = 32 * STATS_SEGS;

template <typename T>
__device__ __forceinline__ void store_op(void* base, int64_t idx, float v);
template <>
__device__ __forceinline__ void store_op<float>(void* base, int64_t idx, float v) {
  static_cast<float*>(base)[idx] = v;
}
template <>
__device__ __forceinline__ void store_op<__nv_bfloat16>(void* base, int64_t idx, float v) {
  static_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
}

// Row scale of an unnormalised address: r = z * (1 / den[row]) when den is given (the addressing
// prologue can hand over z and its row denominators instead of r), 1 otherwise.
__device__ __forceinline__ float row_scale(const float* __restrict__ den, int64_t row) {
  return den ? __frcp_rn(den[row]) : 1.f;
}

// sinv[j] = 1 / den of row t = t_first + j for j <= n (1 everywhere without den; 0 outside [0, T),
// where the tiles hold zeros), filled by the whole CTA
__device__ __forceinline__ void fill_row_scales(float* sinv, const float* __restrict__ den, int b, int T,
                                                int t_first, int n) {
  for (int j = threadIdx.x; j <= n; j += blockDim.x) {
    const int t = t_first + j;
    sinv[j] = den ? ((t >= 0 && t < T) ? __frcp_rn(den[(int64_t)b * T + t]) : 0.f) : 1.f;
  }
}

// largest cluster of the TMA-staged scans (CTAs along T)
constexpr int SCAN_MAX_CLUSTER = 8;

// kernel.py:109-136: k_t = r_{t-1}, c_t = w + sum_{s<=t} lam^(t-s) k_s, q_t = r_t / c_t
template <typename OpT>
__global__ void __launch_bounds__(STATS_THREADS)
    stats_fwd_kernel(const float* __restrict__ r, const float* __restrict__ den, const float* __restrict__ w,
                     const float* __restrict__ g, float* __restrict__ q, float* __restrict__ c,
                     void* __restrict__ qop, void* __restrict__ kop, int64_t ldop, int T, int M) {
  __shared__ float seg_end[STATS_SEGS][32];
  const int lane = threadIdx.x & 31, seg = threadIdx.x >> 5;
  const int b = blockIdx.y;
  const int m = blockIdx.x * 32 + lane;
  const bool valid = m < M;
  const int seg_len = (T + STATS_SEGS - 1) / STATS_SEGS;
  const int t0 = min(T, seg * seg_len), t1 = min(T, t0 + seg_len);
  const float gg = *g;
  const float lam = expf(gg);
  const int64_t row0 = (int64_t)b * T;
  const float* rb = r + row0 * M + m;

  // pass 1: the segment's own decayed sum of k, from a zero carry
  float run = 0.f;
  float kprev = (valid && t0 > 0 && t0 < t1) ? rb[(int64_t)(t0 - 1) * M] * row_scale(den, row0 + t0 - 1) : 0.f;
#pragma unroll 4
  for (int t = t0; t < t1; ++t) {
    const float rt = valid ? rb[(int64_t)t * M] * row_scale(den, row0 + t) : 0.f;
    run = fmaf(lam, run, kprev);
    kprev = rt;
  }
  seg_end[seg][lane] = run;
  __syncthreads();
  float carry = 0.f;
  for (int j = 0; j < seg; ++j) {
    const int len = min(T, (j + 1) * seg_len) - min(T, j * seg_len);
    carry = fmaf(carry, expf(gg * (float)len), seg_end[j][lane]);
  }

  // pass 2: rescan with the carry and write q, c and the operand copies of q and k
  const float wm = valid ? w[m] : 1.f;
  run = carry;
  kprev = (valid && t0 > 0 && t0 < t1) ? rb[(int64_t)(t0 - 1) * M] * row_scale(den, row0 + t0 - 1) : 0.f;
  if (valid) {
#pragma unroll 4
    for (int t = t0; t < t1; ++t) {
      const float rt = rb[(int64_t)t * M] * row_scale(den, row0 + t);
      run = fmaf(lam, run, kprev);
      const float cc = wm + run;
      const float qq = rt / cc;
      const int64_t i = (row0 + t) * M + m;
      q[i] = qq;
      c[i] = cc;
      const int64_t io = (row0 + t) * ldop + m;
      store_op<OpT>(qop, io, qq);
      store_op<OpT>(kop, io, kprev);
      kprev = rt;
    }
  }
}

// kernel.py:139-180 and :232. With dq = dqf + dq_out, walking time backwards:
//   dc_t = -dq_t q_t / c_t,  dkc_t = dc_t + lam dkc_{t+1}  (gradient reaching k through c)
//   dkt_t = dk_t + dkc_t,    dr_t = dq_t / c_t + dkt_{t+1}  (k_{t+1} = r_t)
//   dw += dc_t,  dg += (t - t_mid) (dc (c - w) - k.dkc)                      (through c)
//               dg += (t - t_mid) (q.dqf - k.dk)        (through the fast read, if fast_identity)
// The position weight is centred at t_mid = (T-1)/2: the unweighted sums of q.dqf - k.dk and of
// dc (c - w) - k.dkc are both zero (each pair is the same double sum over (t, s)), so centring
// leaves dg unchanged and keeps the fp32 terms small. The fast-read share by this identity is a
// difference of two large sums of the products' outputs; with bf16 products it loses about one
// digit, so the operator computes that share directly from the scores instead
// (EPI_DECAY_DG in gemm.cu) and runs this kernel with fast_identity = false. Partial sums go to
// `partial` (per batch row and slot for dw; per batch row and slot group for dg, in double) and
// are reduced in a fixed order by the finalize kernels.
__global__ void __launch_bounds__(STATS_THREADS)
    stats_bwd_kernel(const float* __restrict__ dqf, const float* __restrict__ dq_out, const float* __restrict__ dk,
                     const float* __restrict__ q, const float* __restrict__ c, const float* __restrict__ r,
                     const float* __restrict__ den, const float* __restrict__ w, const float* __restrict__ g,
                     float* __restrict__ dr, float* __restrict__ part_dw, double* __restrict__ part_dg, int T, int M,
                     int fast_identity) {
  __shared__ float seg_start[STATS_SEGS][32];
  __shared__ double red_dg[STATS_THREADS];
  __shared__ float red_dw[STATS_SEGS][32];
  const int lane = threadIdx.x & 31, seg = threadIdx.x >> 5;
  const int b = blockIdx.y;
  const int m = blockIdx.x * 32 + lane;
  const bool valid = m < M;
  const int seg_len = (T + STATS_SEGS - 1) / STATS_SEGS;
  const int t0 = min(T, seg * seg_len), t1 = min(T, t0 + seg_len);
  const float gg = *g;
  const float lam = expf(gg);
  const int64_t base = (int64_t)b * T * M + m;
  const bool has_dqo = dq_out != nullptr;

  // pass 1: reverse decayed sum of dc over the segment, from a zero carry
  float run = 0.f;
  if (valid) {
#pragma unroll 4
    for (int t = t1 - 1; t >= t0; --t) {
      const int64_t i = base + (int64_t)t * M;
      const float dq = dqf[i] + (has_dqo ? dq_out[i] : 0.f);
      const float cc = c[i];
      const float dc = -dq * q[i] / cc;
      run = fmaf(lam, run, dc);
    }
  }
  seg_start[seg][lane] = run;
  __syncthreads();
  float carry = 0.f;  // dkc at position t1 (first position after this segment)
  for (int j = STATS_SEGS - 1; j > seg; --j) {
    const int len = min(T, (j + 1) * seg_len) - min(T, j * seg_len);
    carry = fmaf(carry, expf(gg * (float)len), seg_start[j][lane]);
  }

  // pass 2
  const float wm = valid ? w[m] : 0.f;
  const float t_mid = 0.5f * (float)(T - 1);
  double dg_acc = 0.0;
  float dw_acc = 0.f;
  if (valid && t0 < t1) {
    run = carry;
    float dkt_next = (t1 < T) ? dk[base + (int64_t)t1 * M] + carry : 0.f;
#pragma unroll 2
    for (int t = t1 - 1; t >= t0; --t) {
      const int64_t i = base + (int64_t)t * M;
      const float dqfv = dqf[i];
      const float dq = dqfv + (has_dqo ? dq_out[i] : 0.f);
      const float cc = c[i];
      const float qq = q[i];
      const float dc = -dq * qq / cc;
      run = fmaf(lam, run, dc);  // dkc_t
      const float dkv = dk[i];
      const float kt = t > 0 ? r[i - M] * row_scale(den, (int64_t)b * T + t - 1) : 0.f;
      const float dkt = dkv + run;
      dr[i] = dq / cc + dkt_next;
      dkt_next = dkt;
      float term = dc * (cc - wm) - kt * run;
      if (fast_identity) term += qq * dqfv - kt * dkv;
      dg_acc += (double)(((float)t - t_mid) * term);
      dw_acc += dc;
    }
  }
  red_dw[seg][lane] = dw_acc;
  red_dg[threadIdx.x] = dg_acc;
  __syncthreads();
  if (seg == 0) {
    float s = 0.f;
    for (int j = 0; j < STATS_SEGS; ++j) s += red_dw[j][lane];
    if (valid) part_dw[(int64_t)b * M + m] = s;
  }
  for (int stride = STATS_THREADS / 2; stride > 0; stride >>= 1) {
    if (threadIdx.x < stride) red_dg[threadIdx.x] += red_dg[threadIdx.x + stride];
    __syncthreads();
  }
  if (threadIdx.x == 0) part_dg[(int64_t)b * gridDim.x + blockIdx.x] = red_dg[0];
}

namespace cg = cooperative_groups;

// ---- TMA-staged cluster scans --------------------------------------------------------------------
// Same decomposition as above (cluster = 32 slots x whole sequence, CTA = R = WARPS*SEG positions,
// warp = SEG positions, lane = slot), but each CTA first brings its R x 32 tiles of every input
// into shared memory with one TMA bulk-tensor load per array, so the loads need no registers and
// the whole tile is in flight at once. Out-of-range rows and slots arrive as zeros; the write
// address tile (k_t = r_{t-1}) is the r tile loaded one row earlier.

template <int SEG, int WARPS, typename OpT>
__global__ void __launch_bounds__(32 * WARPS)
    stats_fwd_tma_kernel(const __grid_constant__ CUtensorMap map_r, const __grid_constant__ CUtensorMap map_r1,
                         const float* __restrict__ den,
                         const float* __restrict__ w, const float* __restrict__ g, float* __restrict__ q,
                         float* __restrict__ c, void* __restrict__ qop, void* __restrict__ kop, int64_t ldop, int T,
                         int M) {
  pdl_enter();
  constexpr int R = SEG * WARPS;
  // rows cta_t0 - 1 .. cta_t0 + R - 1 of r: row i is the write address k of position cta_t0 + i and
  // the read address of position cta_t0 + i - 1 (R rows in one box, the last row in a second)
  extern __shared__ __align__(128) float tile[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ __align__(8) uint64_t xbar;  // completes when the lower ranks' totals have arrived
  __shared__ float warp_sum[WARPS][32];
  __shared__ float ctot[SCAN_MAX_CLUSTER][32];  // ctot[j]: CTA total of rank j < this rank
  __shared__ float sinv[R + 1];  // row scales of the tile's rows
  __shared__ int ok_flag;
  cg::cluster_group cluster = cg::this_cluster();
  const int C = (int)cluster.num_blocks();
  const int cr = (int)cluster.block_rank();
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const int b = blockIdx.y;
  const int m0 = (blockIdx.x / C) * 32;
  const int m = m0 + lane;
  const int cta_t0 = cr * R;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_init(&xbar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&xbar, (uint32_t)cr * 32u * 4u);
    mbar_arrive_expect_tx(&bar, (R + 1) * 32u * 4u);
    tma_load_3d(&map_r, tile, &bar, m0, cta_t0 - 1, b);
    tma_load_3d(&map_r1, tile + R * 32, &bar, m0, cta_t0 + R - 1, b);
  }
  // the barriers of every CTA are initialised before any CTA sends into them (wait below)
  cluster_arrive_release();
  fill_row_scales(sinv, den, b, T, cta_t0 - 1, R);  // overlaps the tile load
  if (threadIdx.x == 0) ok_flag = 1;
  __syncthreads();
  if (!mbar_wait_bounded(&bar, 0)) {
    raise_device_error(DEVERR_SCAN_TMA_WAIT);
    ok_flag = 0;
  }
  __syncthreads();
  const bool ok = ok_flag != 0;
  const float gg = *g;
  const float lam = expf(gg);
  const float* xt = tile + (wp * SEG) * 32 + lane;  // xt[i * 32]: k of position t0 + i, r of t0 + i - 1
  const float* si = sinv + wp * SEG;
  float run = 0.f;
  if (ok) {
#pragma unroll
    for (int i = 0; i < SEG; ++i) run = fmaf(lam, run, xt[i * 32] * si[i]);
  }
  warp_sum[wp][lane] = run;
  __syncthreads();
  const float lam_seg = expf(gg * (float)SEG);
  cluster_wait_acquire();
  if (wp == 0) {
    // this CTA's total goes straight into the shared memory of every higher rank
    float tot = 0.f;
    for (int j = 0; j < WARPS; ++j) tot = fmaf(tot, lam_seg, warp_sum[j][lane]);
    const uint32_t slot = smem_u32(&ctot[cr][lane]), xb = smem_u32(&xbar);
    for (int j = cr + 1; j < C; ++j) st_async_f32(mapa_shared(slot, j), tot, mapa_shared(xb, j));
  }
  const float lam_cta = expf(gg * (float)R);
  float carry = 0.f;
  if (cr > 0 && !mbar_wait_bounded(&xbar, 0)) raise_device_error(DEVERR_SCAN_TMA_WAIT);
  for (int j = 0; j < cr; ++j) carry = fmaf(carry, lam_cta, ctot[j][lane]);
  for (int j = 0; j < wp; ++j) carry = fmaf(carry, lam_seg, warp_sum[j][lane]);
  if (ok && m < M) {
    const float wm = w[m];
    const int t0 = cta_t0 + wp * SEG;
    const int64_t row = (int64_t)b * T + t0;
    float* qp = q ? q + row * M + m : nullptr;
    float* cp = c ? c + row * M + m : nullptr;
    const int64_t io = row * ldop + m;
    run = carry;
    float kk = xt[0] * si[0];
#pragma unroll
    for (int i = 0; i < SEG; ++i) {
      const float rv = xt[(i + 1) * 32] * si[i + 1];
      if (t0 + i < T) {
        run = fmaf(lam, run, kk);
        const float cc = wm + run;
        const float qq = rv * fast_rcp(cc);
        if (qp) qp[(int64_t)i * M] = qq;
        if (cp) cp[(int64_t)i * M] = cc;
        store_op<OpT>(qop, io + (int64_t)i * ldop, qq);
        store_op<OpT>(kop, io + (int64_t)i * ldop, kk);
      }
      kk = rv;
    }
  }
}

// RECOMPUTE: instead of reading the saved q and c (two fp32 arrays), rebuild them from the r tile
// (loaded one row earlier and one row longer, so it holds both k_t = r_{t-1} and r_t) by running the
// forward scan again with the same segment structure as stats_fwd_tma_kernel: identical c, q.
template <int SEG, int WARPS, bool RECOMPUTE>
__global__ void __launch_bounds__(32 * WARPS)
    stats_bwd_tma_kernel(const __grid_constant__ CUtensorMap map_dqf, const __grid_constant__ CUtensorMap map_dqo,
                         const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_c,
                         const __grid_constant__ CUtensorMap map_dk, const __grid_constant__ CUtensorMap map_r,
                         const float* __restrict__ dk, const float* __restrict__ den, const float* __restrict__ w,
                         const float* __restrict__ g, float* __restrict__ dr, float* __restrict__ part_dw,
                         double* __restrict__ part_dg, int T, int M, int has_dqo, int fast_identity) {
  pdl_enter();
  constexpr int R = SEG * WARPS;
  constexpr int TILE = R * 32;
  // tiles: dqf, dk, then either the r tile rows t0-1 .. t0+R-1 (recompute) or q, c, k (saved),
  // then dq_out when given
  extern __shared__ __align__(128) float tile[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ float warp_sum[WARPS][32];
  __shared__ float warp_dw[WARPS][32];
  __shared__ __align__(8) uint64_t xbar_f;  // lower ranks' forward totals have arrived (recompute)
  __shared__ __align__(8) uint64_t xbar_r;  // higher ranks' reverse totals have arrived
  __shared__ float ctot_f[SCAN_MAX_CLUSTER][32];
  __shared__ float ctot_r[SCAN_MAX_CLUSTER][32];
  __shared__ double red_dg[32 * WARPS];
  __shared__ float sinv[R + 1];  // row scales of the r tile's rows cta_t0 - 1 .. cta_t0 + R - 1
  __shared__ int ok_flag;
  cg::cluster_group cluster = cg::this_cluster();
  const int C = (int)cluster.num_blocks();
  const int cr = (int)cluster.block_rank();
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const int b = blockIdx.y;
  const int m0 = (blockIdx.x / C) * 32;
  const int m = m0 + lane;
  const bool valid = m < M;
  const int cta_t0 = cr * R;
  float* t_dqf = tile;
  float* t_dk = tile + TILE;
  float* t_x = tile + 2 * TILE;  // recompute: r rows (R+1); saved: q, c, k tiles
  float* t_dqo = t_x + (RECOMPUTE ? R + 1 : 3 * R) * 32;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_init(&xbar_f, 1);
    mbar_init(&xbar_r, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&xbar_f, RECOMPUTE ? (uint32_t)cr * 128u : 0u);
    mbar_arrive_expect_tx(&xbar_r, (uint32_t)(C - 1 - cr) * 128u);
    const uint32_t bytes = ((has_dqo ? 3u : 2u) * TILE + (RECOMPUTE ? (uint32_t)(R + 1) * 32u : 3u * TILE)) * 4u;
    mbar_arrive_expect_tx(&bar, bytes);
    tma_load_3d(&map_dqf, t_dqf, &bar, m0, cta_t0, b);
    if (has_dqo) tma_load_3d(&map_dqo, t_dqo, &bar, m0, cta_t0, b);
    tma_load_3d(&map_dk, t_dk, &bar, m0, cta_t0, b);
    if (RECOMPUTE) {
      tma_load_3d(&map_r, t_x, &bar, m0, cta_t0 - 1, b);
    } else {
      tma_load_3d(&map_q, t_x, &bar, m0, cta_t0, b);
      tma_load_3d(&map_c, t_x + TILE, &bar, m0, cta_t0, b);
      tma_load_3d(&map_r, t_x + 2 * TILE, &bar, m0, cta_t0 - 1, b);
    }
    ok_flag = 1;
  }
  // the barriers of every CTA are initialised before any CTA sends into them (wait below)
  cluster_arrive_release();
  fill_row_scales(sinv, den, b, T, cta_t0 - 1, R);  // overlaps the tile loads
  __syncthreads();
  if (!mbar_wait_bounded(&bar, 0)) {
    raise_device_error(DEVERR_SCAN_TMA_WAIT);
    ok_flag = 0;
  }
  __syncthreads();
  const bool ok = ok_flag != 0;
  const float gg = *g;
  const float lam = expf(gg);
  const float lam_seg = expf(gg * (float)SEG);
  const float lam_cta = expf(gg * (float)R);
  const float wm = valid ? w[m] : 0.f;
  const float t_mid = 0.5f * (float)(T - 1);
  const int t0 = cta_t0 + wp * SEG;
  const int o = (wp * SEG) * 32 + lane;
  const float* s_dqf = t_dqf + o;
  const float* s_dqo = t_dqo + o;
  const float* s_dk = t_dk + o;
  const float* s_k = RECOMPUTE ? t_x + o : t_x + 2 * TILE + o;   // k_t = r_{t-1}
  const float* s_r = t_x + o + 32;                                // recompute: r_t
  const float* s_q = t_x + o;                                     // saved q
  const float* s_c = t_x + TILE + o;                              // saved c
  const float* si = sinv + wp * SEG;  // si[i]: scale of k row i, si[i + 1]: of r row i

  float n_carry = 0.f;
  if (RECOMPUTE) {
    // forward scan of k, exactly as stats_fwd_tma_kernel does it, to rebuild n_t
    float run = 0.f;
    if (ok) {
#pragma unroll
      for (int i = 0; i < SEG; ++i) run = fmaf(lam, run, s_k[i * 32] * si[i]);
    }
    warp_sum[wp][lane] = run;
    __syncthreads();
    cluster_wait_acquire();
    if (wp == 0) {
      float tot = 0.f;
      for (int j = 0; j < WARPS; ++j) tot = fmaf(tot, lam_seg, warp_sum[j][lane]);
      const uint32_t slot = smem_u32(&ctot_f[cr][lane]), xb = smem_u32(&xbar_f);
      for (int j = cr + 1; j < C; ++j) st_async_f32(mapa_shared(slot, j), tot, mapa_shared(xb, j));
    }
    if (cr > 0 && !mbar_wait_bounded(&xbar_f, 0)) raise_device_error(DEVERR_SCAN_TMA_WAIT);
    for (int j = 0; j < cr; ++j) n_carry = fmaf(n_carry, lam_cta, ctot_f[j][lane]);
    for (int j = 0; j < wp; ++j) n_carry = fmaf(n_carry, lam_seg, warp_sum[j][lane]);
    __syncthreads();  // warp_sum is reused below
  } else {
    cluster_wait_acquire();
  }

  float dw_acc = 0.f, dg_f = 0.f, run = 0.f;
  float drd_v[SEG], dc_v[SEG];  // dq / c and dc per row, kept for the reverse pass
  if (ok) {
    float n = n_carry;
#pragma unroll
    for (int i = 0; i < SEG; ++i) {
      const int t = t0 + i;
      float cc, qq;
      float inv;
      if (RECOMPUTE) {
        n = fmaf(lam, n, s_k[i * 32] * si[i]);
        cc = wm + n;
        inv = fast_rcp(cc);
        qq = (s_r[i * 32] * si[i + 1]) * inv;
      } else {
        cc = s_c[i * 32];
        qq = s_q[i * 32];
        inv = fast_rcp(cc);
      }
      if (!(t < T && valid)) {
        cc = 1.f;
        qq = 0.f;
        inv = 1.f;
      }
      const float dqfv = s_dqf[i * 32];
      const float dq = dqfv + (has_dqo ? s_dqo[i * 32] : 0.f);
      const float drd = dq * inv;
      const float dc = -drd * qq;
      drd_v[i] = drd;
      dc_v[i] = dc;
      dw_acc += dc;
      float term = dc * (cc - wm);
      if (fast_identity) term += qq * dqfv;
      dg_f = fmaf((float)t - t_mid, term, dg_f);
    }
#pragma unroll
    for (int i = SEG - 1; i >= 0; --i) run = fmaf(lam, run, dc_v[i]);
  } else {
#pragma unroll
    for (int i = 0; i < SEG; ++i) drd_v[i] = dc_v[i] = 0.f;
  }
  warp_sum[wp][lane] = run;
  warp_dw[wp][lane] = dw_acc;
  __syncthreads();
  if (wp == 0) {
    // this CTA's reverse total goes into the shared memory of every lower rank
    float tot = 0.f;
    for (int j = WARPS - 1; j >= 0; --j) tot = fmaf(tot, lam_seg, warp_sum[j][lane]);
    const uint32_t slot = smem_u32(&ctot_r[cr][lane]), xb = smem_u32(&xbar_r);
    for (int j = 0; j < cr; ++j) st_async_f32(mapa_shared(slot, j), tot, mapa_shared(xb, j));
  }
  if (cr < C - 1 && !mbar_wait_bounded(&xbar_r, 0)) raise_device_error(DEVERR_SCAN_TMA_WAIT);
  float carry = 0.f;  // dkc at position t0 + SEG
  for (int j = C - 1; j > cr; --j) carry = fmaf(carry, lam_cta, ctot_r[j][lane]);
  for (int j = WARPS - 1; j > wp; --j) carry = fmaf(carry, lam_seg, warp_sum[j][lane]);
  double dg_acc = (double)dg_f;
  if (ok && valid) {
    const int64_t base = (int64_t)b * T * M + m;
    const int t_end = t0 + SEG;
    float dk_end = 0.f;
    if (t_end < T) dk_end = (wp + 1 < WARPS) ? s_dk[SEG * 32] : dk[base + (int64_t)t_end * M];
    float dkt_next = (t_end < T) ? dk_end + carry : 0.f;
    run = carry;
    float dg_s = 0.f;
#pragma unroll
    for (int i = SEG - 1; i >= 0; --i) {
      const int t = t0 + i;
      if (t < T) {
        const float dkv = s_dk[i * 32];
        const float kv = s_k[i * 32] * si[i];
        run = fmaf(lam, run, dc_v[i]);  // dkc_t
        dr[base + (int64_t)t * M] = drd_v[i] + dkt_next;
        dkt_next = dkv + run;
        float term = -kv * run;
        if (fast_identity) term -= kv * dkv;
        dg_s = fmaf((float)t - t_mid, term, dg_s);
      }
    }
    dg_acc += (double)dg_s;
  }
  if (wp == 0 && valid) {
    float s2 = 0.f;
    for (int j = 0; j < WARPS; ++j) s2 += warp_dw[j][lane];
    part_dw[((int64_t)b * C + cr) * M + m] = s2;
  }
  red_dg[threadIdx.x] = dg_acc;
  __syncthreads();
  for (int stride = 16 * WARPS; stride > 0; stride >>= 1) {
    if ((int)threadIdx.x < stride) red_dg[threadIdx.x] += red_dg[threadIdx.x + stride];
    __syncthreads();
  }
  if (threadIdx.x == 0) part_dg[(int64_t)b * gridDim.x + blockIdx.x] = red_dg[0];
}

// ---- persistent, pipelined cluster scans ---------------------------------------------------------
// The kernels above give every (batch row, 32 slots) item its own cluster: a CTA loads its tiles,
// scans, exchanges carries and stores, so its loads never overlap its own compute. Here a cluster
// of C CTAs (C = cdiv(T, R)) stays resident and walks a list of items (item = batch row b and slot
// block m0; cluster k takes items k, k + G, k + 2G, ... for G clusters), with the TMA loads of the
// next STAGES - 1 items in flight while the current one is scanned. Per item the arithmetic is that
// of the kernels above, in the same order (identical results). Carry slots are reused from item to
// item. In the backward a rank cannot run ahead of the peers it exchanges with: its next forward
// total waits for their reverse totals of the current item and vice versa, and two slots per
// direction (alternating by item) keep every slot unread-safe. The forward has no reply, so after
// reading its carries (and a CTA barrier) each CTA arrives on the cluster barrier, relaxed, and
// waits on it before its next send.
// Each exchange mbarrier is armed (expect_tx) before any total of its item can be sent, and re-armed
// for its next use only after every thread of the CTA has passed the wait on the current one.
// Every mbarrier wait is bounded; after a timeout the CTA records the error and keeps the protocol
// going with short limits, so its peers are never left waiting.

constexpr uint64_t SCAN_SHORT_WAIT_NS = 10000000ull;  // waits after an error: 10 ms
constexpr int SCAN_RING = 4;  // dealt items in flight per CTA of the forward scan

// Row scales of the next item, in two steps so that the global load's latency overlaps the current
// item: thread i (i <= n) loads den of row t_first + i early (den_prefetch) and stores the scale
// later (den_store): 1 / den, or 1 without den, 0 outside [0, T), as fill_row_scales.
__device__ __forceinline__ float den_prefetch(const float* __restrict__ den, int b, int T, int t_first, int n) {
  const int i = threadIdx.x, t = t_first + i;
  return (den && i <= n && t >= 0 && t < T) ? den[(int64_t)b * T + t] : 0.f;
}
__device__ __forceinline__ void den_store(float* sinv, const float* den, float dv, int T, int t_first, int n) {
  const int i = threadIdx.x, t = t_first + i;
  if (i <= n) sinv[i] = den ? ((t >= 0 && t < T) ? __frcp_rn(dv) : 0.f) : 1.f;
}

// Two slots of one item as a pair of floats (8-byte stores; the bf16 operand pair packed in 4 bytes).
template <typename T>
__device__ __forceinline__ void store_op2(void* base, int64_t idx, float2 v);
template <>
__device__ __forceinline__ void store_op2<float>(void* base, int64_t idx, float2 v) {
  *reinterpret_cast<float2*>(static_cast<float*>(base) + idx) = v;
}
template <>
__device__ __forceinline__ void store_op2<__nv_bfloat16>(void* base, int64_t idx, float2 v) {
  *reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(base) + idx) = __floats2bfloat162_rn(v.x, v.y);
}

// Forward scan (kernel.py:109-136) on the TMA-staged r tile of one item per stage. Each warp owns
// SEG consecutive rows of the CTA's R; a thread holds two adjacent slots of SEG / 2 of those rows
// (lanes 0-15 the first half, lanes 16-31 the second), so every shared-memory load and global
// store moves two slots. The warp's total is the second half's plus lam^(SEG/2) times the first's.
// Items: a cluster's first STAGES items are fixed (k0, k0 + G, ...); with `tickets` the rest are
// handed out in arrival order by rank 0 of each cluster (a global ticket, sent to every rank of the
// cluster through shared memory), so clusters that run faster take more items; without, every
// item is fixed (k0 + j G).
template <int SEG, int WARPS, int STAGES, typename OpT>
__global__ void __launch_bounds__(32 * WARPS, 6)  // six CTAs per SM: <= 40 registers
    stats_fwd_pipe_kernel(const __grid_constant__ CUtensorMap map_r, const __grid_constant__ CUtensorMap map_r1,
                          const float* __restrict__ den, const float* __restrict__ w, const float* __restrict__ g,
                          float* __restrict__ q, float* __restrict__ c, void* __restrict__ qop,
                          void* __restrict__ kop, int64_t ldop, int B, int T, int M,
                          unsigned int* __restrict__ tickets) {
  pdl_enter();
  static_assert(SEG % 2 == 0, "two half-segments per warp");
  constexpr int R = SEG * WARPS;
  constexpr int H = SEG / 2;
  constexpr int STAGE_FLOATS = (R + 1) * 32;
  extern __shared__ __align__(128) float tile[];
  __shared__ __align__(8) uint64_t full[STAGES];
  __shared__ __align__(8) uint64_t xbar;
  __shared__ __align__(16) float warp_sum[WARPS][32];
  __shared__ __align__(16) float ctot[SCAN_MAX_CLUSTER][32];
  __shared__ float sinv[2][R + 1];  // row scales of the current and the next item
  __shared__ int ok_flag;
  __shared__ int ring_item[SCAN_RING];  // items of iterations STAGES, STAGES + 1, ... (use u: slot u % SCAN_RING)
  __shared__ __align__(8) uint64_t ring_bar[SCAN_RING];
  __shared__ int dealt[SCAN_RING];  // the same items, stored by thread 0 once received: read after a CTA barrier
  static_assert(32 * WARPS > R, "one thread per row scale");
  static_assert(SCAN_RING >= STAGES + 2, "rank 0 runs at most one item ahead of its peers");
  cg::cluster_group cluster = cg::this_cluster();
  const int C = (int)cluster.num_blocks();
  const int cr = (int)cluster.block_rank();
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const int half = lane >> 4, s2 = (lane & 15) * 2;  // rows [half * H, half * H + H) of the warp; slots s2, s2 + 1
  const int cta_t0 = cr * R;
  const int nmb = (M + 31) / 32;
  const int n_items = B * nmb;
  const int G = (int)gridDim.x / C;
  const int k0 = (int)blockIdx.x / C;
  // item of iteration j. Thread 0 stores a dealt item (use j - STAGES) at the end of iteration
  // j - STAGES; the other threads read it only after the next CTA barrier: as the current item at the
  // top of iteration j, as the next item after the first barrier of iteration j - 1.
  auto item_of = [&](int j) -> int {
    return (j < STAGES || !tickets) ? k0 + j * G : dealt[(j - STAGES) % SCAN_RING];
  };
  auto issue = [&](int j, int item) {
    if (item >= n_items) return;
    const int bb = item / nmb, mm0 = (item % nmb) * 32;
    float* st = tile + (j % STAGES) * STAGE_FLOATS;
    uint64_t* bar = &full[j % STAGES];
    mbar_arrive_expect_tx(bar, (uint32_t)STAGE_FLOATS * 4u);
    tma_load_3d(&map_r, st, bar, mm0, cta_t0 - 1, bb);
    tma_load_3d(&map_r1, st + R * 32, bar, mm0, cta_t0 + R - 1, bb);
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1);
    mbar_init(&xbar, 1);
    for (int s = 0; s < SCAN_RING; ++s) mbar_init(&ring_bar[s], 1);
    fence_barrier_init();
    if (cr > 0) mbar_arrive_expect_tx(&xbar, (uint32_t)cr * 128u);  // armed for the first item
    for (int s = 0; s < SCAN_RING; ++s) mbar_arrive_expect_tx(&ring_bar[s], 4u);  // armed for uses 0 .. SCAN_RING - 1
    ok_flag = 1;
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int j = 0; j < STAGES; ++j) issue(j, k0 + j * G);
  bool dealt_out = false;  // rank 0, thread 0: the ticket ran past the last item
  // the barriers of every CTA are initialised before any CTA sends into them
  __syncwarp();
  cluster_sync_all();
  const float gg = *g;
  const float lam = expf(gg);
  const float lam_h = expf(gg * (float)H);
  const float lam_seg = expf(gg * (float)SEG);
  const float lam_cta = expf(gg * (float)R);
  // prior masses of this thread's two slots (the current and the next item)
  auto load_w = [&](int item) {
    const int m0 = (item % nmb) * 32 + s2;
    return m0 < M ? make_float2(w[m0], w[m0 + 1]) : make_float2(0.f, 0.f);  // M % 4 == 0: both or neither
  };
  float2 w_cur = make_float2(0.f, 0.f);
  if (k0 < n_items) {
    w_cur = load_w(k0);
    den_store(sinv[0], den, den_prefetch(den, k0 / nmb, T, cta_t0 - 1, R), T, cta_t0 - 1, R);
  }
  for (int j = 0;; ++j) {
    const int item = item_of(j);
    if (item >= n_items) break;
    const int b = item / nmb;
    const int m0 = (item % nmb) * 32 + s2;
    const float* xs = tile + (j % STAGES) * STAGE_FLOATS;
    const uint64_t lim = ok_flag ? 2000000000ull : SCAN_SHORT_WAIT_NS;
    if (!mbar_wait_bounded(&full[j % STAGES], (uint32_t)(j / STAGES) & 1u, lim)) {
      raise_device_error(DEVERR_SCAN_TMA_WAIT);
      ok_flag = 0;
    }
    __syncthreads();  // also orders thread 0's store of the next item (end of the previous iteration)
    // the next item's row scales and prior masses: loaded now, used after this item
    const int item_n = item_of(j + 1);
    const bool has_next = item_n < n_items;
    const float den_n = has_next ? den_prefetch(den, item_n / nmb, T, cta_t0 - 1, R) : 0.f;
    const float2 w_n = has_next ? load_w(item_n) : make_float2(0.f, 0.f);
    // xt[i * 32]: k of position t0 + i (the r row before it), xt[(i + 1) * 32]: r of t0 + i
    const int rh = wp * SEG + half * H;
    const float* xt = xs + rh * 32 + s2;
    const float* si = sinv[j & 1] + rh;
    float2 run = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < H; ++i) {
      const float2 k2 = *reinterpret_cast<const float2*>(xt + i * 32);
      const float sv = si[i];
      run.x = fmaf(lam, run.x, k2.x * sv);
      run.y = fmaf(lam, run.y, k2.y * sv);
    }
    // the first half's total, seen by the second half's lanes of the same slots
    const float lo_x = __shfl_sync(0xffffffffu, run.x, lane & 15);
    const float lo_y = __shfl_sync(0xffffffffu, run.y, lane & 15);
    if (half) *reinterpret_cast<float2*>(&warp_sum[wp][s2]) = make_float2(fmaf(lam_h, lo_x, run.x), fmaf(lam_h, lo_y, run.y));
    __syncthreads();
    __syncwarp();
    if (j > 0) cluster_wait_acquire();  // every CTA has read the previous item's totals
    if (wp == 0) {
      float tot = 0.f;
      for (int jj = 0; jj < WARPS; ++jj) tot = fmaf(tot, lam_seg, warp_sum[jj][lane]);
      const uint32_t slot = smem_u32(&ctot[cr][lane]), xb = smem_u32(&xbar);
      for (int jj = cr + 1; jj < C; ++jj) st_async_f32(mapa_shared(slot, jj), tot, mapa_shared(xb, jj));
    }
    if (cr > 0) {
      if (!mbar_wait_bounded(&xbar, (uint32_t)j & 1u, ok_flag ? 2000000000ull : SCAN_SHORT_WAIT_NS)) {
        raise_device_error(DEVERR_SCAN_TMA_WAIT);
        ok_flag = 0;
      }
      // armed for the next item: its totals are sent only after this CTA's cluster arrive below
      if (threadIdx.x == 0) mbar_arrive_expect_tx(&xbar, (uint32_t)cr * 128u);
    }
    float2 carry = make_float2(0.f, 0.f);
    // unrolled to the static bounds so that the shared-memory loads issue together
#pragma unroll
    for (int jj = 0; jj < SCAN_MAX_CLUSTER; ++jj)
      if (jj < cr) {
        const float2 t2 = *reinterpret_cast<const float2*>(&ctot[jj][s2]);
        carry.x = fmaf(carry.x, lam_cta, t2.x);
        carry.y = fmaf(carry.y, lam_cta, t2.y);
      }
#pragma unroll
    for (int jj = 0; jj < WARPS; ++jj)
      if (jj < wp) {
        const float2 t2 = *reinterpret_cast<const float2*>(&warp_sum[jj][s2]);
        carry.x = fmaf(carry.x, lam_seg, t2.x);
        carry.y = fmaf(carry.y, lam_seg, t2.y);
      }
    if (half) {  // the second half starts after the first half's rows
      carry.x = fmaf(lam_h, carry.x, lo_x);
      carry.y = fmaf(lam_h, carry.y, lo_y);
    }
    // this CTA's totals slots may be written again: every thread has read them (the CTA barrier),
    // so the arrive needs no release ordering (which would also wait for the previous item's stores)
    __syncthreads();
    cluster_arrive_relaxed();
    if (m0 < M) {
      const float2 wm = w_cur;
      const int t0 = cta_t0 + rh;
      const int64_t row = (int64_t)b * T + t0;
      float* qp = q ? q + row * M + m0 : nullptr;
      float* cp = c ? c + row * M + m0 : nullptr;
      const int64_t io = row * ldop + m0;
      run = carry;
      const float2 k0v = *reinterpret_cast<const float2*>(xt);
      float2 kk = make_float2(k0v.x * si[0], k0v.y * si[0]);
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const float2 r2 = *reinterpret_cast<const float2*>(xt + (i + 1) * 32);
        const float sv = si[i + 1];
        const float2 rv = make_float2(r2.x * sv, r2.y * sv);
        if (t0 + i < T) {
          run.x = fmaf(lam, run.x, kk.x);
          run.y = fmaf(lam, run.y, kk.y);
          const float2 cc = make_float2(wm.x + run.x, wm.y + run.y);
          const float2 qq = make_float2(rv.x * fast_rcp(cc.x), rv.y * fast_rcp(cc.y));
          if (qp) *reinterpret_cast<float2*>(qp + (int64_t)i * M) = qq;
          if (cp) *reinterpret_cast<float2*>(cp + (int64_t)i * M) = cc;
          store_op2<OpT>(qop, io + (int64_t)i * ldop, qq);
          store_op2<OpT>(kop, io + (int64_t)i * ldop, kk);
        }
        kk = rv;
      }
    }
    if (has_next) den_store(sinv[(j + 1) & 1], den, den_n, T, cta_t0 - 1, R);  // last read in item j - 1
    w_cur = w_n;
    __syncthreads();  // the stage, sinv[j & 1] and warp_sum are free again
    if (threadIdx.x == 0) {
      int it = k0 + (j + STAGES) * G;
      if (tickets) {  // ring use j: the item of iteration j + STAGES
        const int sl = j % SCAN_RING;
        if (cr == 0) {  // rank 0 deals: the next ticket, to every rank of the cluster
          int v = n_items;
          if (!dealt_out) {
            v = STAGES * G + (int)atomicAdd(&tickets[0], 1u);
            if (v >= n_items) {
              v = n_items;
              dealt_out = true;
              // the last cluster to run out resets the pair for a later launch
              if (atomicAdd(&tickets[1], 1u) == (unsigned)(G - 1)) {
                atomicExch(&tickets[0], 0u);
                atomicExch(&tickets[1], 0u);
              }
            }
          }
          const uint32_t slot = smem_u32(&ring_item[sl]), rb = smem_u32(&ring_bar[sl]);
          for (int jj = 0; jj < C; ++jj) st_async_f32(mapa_shared(slot, jj), __int_as_float(v), mapa_shared(rb, jj));
        }
        it = n_items;
        if (mbar_wait_bounded(&ring_bar[sl], (uint32_t)(j / SCAN_RING) & 1u, ok_flag ? 2000000000ull : SCAN_SHORT_WAIT_NS)) {
          it = ring_item[sl];
          if (it != n_items && (it < STAGES * G || it > n_items)) {  // neither a dealt item nor the end mark
            raise_device_error(DEVERR_SCAN_TMA_WAIT);
            ok_flag = 0;
            it = n_items;
          }
        } else {
          raise_device_error(DEVERR_SCAN_TMA_WAIT);
          ok_flag = 0;
        }
        dealt[sl] = it;
        mbar_arrive_expect_tx(&ring_bar[sl], 4u);  // armed for use j + SCAN_RING
      }
      fence_proxy_async_smem();
      issue(j + STAGES, it);
    }
  }
  // pairs the last arrive; no CTA leaves while a peer may still send into its shared memory
  __syncwarp();
  if (k0 < n_items) cluster_wait_acquire();
}

// Backward with q and c rebuilt from the r tile (kernel.py:139-180 and the shift-add of :232).
// Stage layout: dqf (R rows), dk (R + 1 rows), r (R + 1 rows from position cta_t0 - 1), dq_out (R
// rows, when given). part_dg gets one partial per CTA (its items' sum); part_dw one row per (b, rank).
// As in the forward, a thread holds two adjacent slots of half of its warp's SEG rows; the halves are
// joined with lam^(SEG/2): the first half's forward total carried into the second half, the second
// half's reverse total into the first.
template <int SEG, int WARPS, int STAGES>
__global__ void __launch_bounds__(32 * WARPS, 2)
    stats_bwd_pipe_kernel(const __grid_constant__ CUtensorMap map_dqf, const __grid_constant__ CUtensorMap map_dqo,
                          const __grid_constant__ CUtensorMap map_dk, const __grid_constant__ CUtensorMap map_r,
                          const float* __restrict__ den, const float* __restrict__ w, const float* __restrict__ g,
                          float* __restrict__ dr, float* __restrict__ part_dw, double* __restrict__ part_dg, int B,
                          int T, int M, int has_dqo, int fast_identity) {
  pdl_enter();
  static_assert(SEG % 2 == 0, "two half-segments per warp");
  constexpr int R = SEG * WARPS;
  constexpr int H = SEG / 2;
  constexpr int TILE = R * 32;
  extern __shared__ __align__(128) float tile[];
  __shared__ __align__(8) uint64_t full[STAGES];
  __shared__ __align__(8) uint64_t xbar_f[2];  // lower ranks' forward totals of the item have arrived
  __shared__ __align__(8) uint64_t xbar_r[2];  // higher ranks' reverse totals have arrived
  __shared__ __align__(16) float warp_sum[WARPS][32];     // reverse partial sums of the current item
  __shared__ __align__(16) float warp_sum_f[2][WARPS][32];  // forward partial sums, by item parity
  __shared__ __align__(16) float warp_dw[WARPS][32];
  __shared__ __align__(16) float ctot_f[2][SCAN_MAX_CLUSTER][32];
  __shared__ __align__(16) float ctot_r[2][SCAN_MAX_CLUSTER][32];
  __shared__ double red_dg[32 * WARPS];
  __shared__ float sinv[2][R + 1];  // row scales of the current and the next item
  __shared__ int ok_flag;
  static_assert(32 * WARPS > R, "one thread per row scale");
  cg::cluster_group cluster = cg::this_cluster();
  const int C = (int)cluster.num_blocks();
  const int cr = (int)cluster.block_rank();
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const int half = lane >> 4, s2 = (lane & 15) * 2;  // rows [half * H, half * H + H) of the warp; slots s2, s2 + 1
  const int rh = wp * SEG + half * H;                // this thread's first row within the CTA's R
  const int cta_t0 = cr * R;
  const int nmb = (M + 31) / 32;
  const int n_items = B * nmb;
  const int G = (int)gridDim.x / C;
  const int k0 = (int)blockIdx.x / C;
  const int stage_floats = (3 * R + 2 + (has_dqo ? R : 0)) * 32;
  auto issue = [&](int j) {
    const int item = k0 + j * G;
    if (item >= n_items) return;
    const int bb = item / nmb, mm0 = (item % nmb) * 32;
    float* st = tile + (j % STAGES) * stage_floats;
    uint64_t* bar = &full[j % STAGES];
    mbar_arrive_expect_tx(bar, (uint32_t)stage_floats * 4u);
    tma_load_3d(&map_dqf, st, bar, mm0, cta_t0, bb);
    tma_load_3d(&map_dk, st + TILE, bar, mm0, cta_t0, bb);  // R + 1 rows: the next CTA's first one too
    tma_load_3d(&map_r, st + 2 * TILE + 32, bar, mm0, cta_t0 - 1, bb);
    if (has_dqo) tma_load_3d(&map_dqo, st + 3 * TILE + 64, bar, mm0, cta_t0, bb);
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&xbar_f[s], 1);
      mbar_init(&xbar_r[s], 1);
    }
    fence_barrier_init();
    // armed for the first two items; each is re-armed for the item after next once read
    for (int s = 0; s < 2; ++s) {
      if (cr > 0) mbar_arrive_expect_tx(&xbar_f[s], (uint32_t)cr * 128u);
      if (cr < C - 1) mbar_arrive_expect_tx(&xbar_r[s], (uint32_t)(C - 1 - cr) * 128u);
    }
    ok_flag = 1;
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int j = 0; j < STAGES; ++j) issue(j);
  // the barriers of every CTA are initialised before any CTA sends into them
  __syncwarp();
  cluster_sync_all();
  const float gg = *g;
  const float lam = expf(gg);
  const float lam_h = expf(gg * (float)H);
  const float lam_seg = expf(gg * (float)SEG);
  const float lam_cta = expf(gg * (float)R);
  const float t_mid = 0.5f * (float)(T - 1);
  const int t0 = cta_t0 + rh;
  const int o = rh * 32 + s2;
  double dg_acc = 0.0;
  auto load_w = [&](int item) {
    const int m0 = (item % nmb) * 32 + s2;
    return m0 < M ? make_float2(w[m0], w[m0 + 1]) : make_float2(0.f, 0.f);  // M % 4 == 0: both or neither
  };
  float2 w_cur = make_float2(0.f, 0.f);
  float2 lo_cur = make_float2(0.f, 0.f);  // the first half's forward total of the current item
  // Forward part of item jn: wait for its tile, rescan the write addresses k of this CTA's rows from
  // zero (warp_sum_f) and send the CTA's total into the higher ranks' slot jn & 1; returns the first
  // half's total for the second half's lanes. Item jn + 1's forward part runs during item jn (after
  // its reverse totals are sent), so the forward exchange is complete by the time item jn + 1 needs it.
  auto forward_part = [&](int jn) -> float2 {
    if (!mbar_wait_bounded(&full[jn % STAGES], (uint32_t)(jn / STAGES) & 1u,
                           ok_flag ? 2000000000ull : SCAN_SHORT_WAIT_NS)) {
      raise_device_error(DEVERR_SCAN_TMA_WAIT);
      ok_flag = 0;
    }
    __syncthreads();  // the tile and this item's row scales are visible to every thread
    const float* s_kn = tile + (jn % STAGES) * stage_floats + 2 * TILE + 32 + o;
    const float* sin = sinv[jn & 1] + rh;
    float2 run = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < H; ++i) {
      const float2 k2 = *reinterpret_cast<const float2*>(s_kn + i * 32);
      const float sv = sin[i];
      run.x = fmaf(lam, run.x, k2.x * sv);
      run.y = fmaf(lam, run.y, k2.y * sv);
    }
    const float2 lo = make_float2(__shfl_sync(0xffffffffu, run.x, lane & 15), __shfl_sync(0xffffffffu, run.y, lane & 15));
    if (half)
      *reinterpret_cast<float2*>(&warp_sum_f[jn & 1][wp][s2]) = make_float2(fmaf(lam_h, lo.x, run.x), fmaf(lam_h, lo.y, run.y));
    __syncthreads();
    if (wp == 0) {
      float tot = 0.f;
      for (int jj = 0; jj < WARPS; ++jj) tot = fmaf(tot, lam_seg, warp_sum_f[jn & 1][jj][lane]);
      const uint32_t slot = smem_u32(&ctot_f[jn & 1][cr][lane]), xb = smem_u32(&xbar_f[jn & 1]);
      for (int jj = cr + 1; jj < C; ++jj) st_async_f32(mapa_shared(slot, jj), tot, mapa_shared(xb, jj));
    }
    return lo;
  };
  if (k0 < n_items) {
    w_cur = load_w(k0);
    den_store(sinv[0], den, den_prefetch(den, k0 / nmb, T, cta_t0 - 1, R), T, cta_t0 - 1, R);
    lo_cur = forward_part(0);
  }
  for (int j = 0;; ++j) {
    const int item = k0 + j * G;
    if (item >= n_items) break;
    const int b = item / nmb;
    const int m0 = (item % nmb) * 32 + s2;
    const bool valid = m0 < M;
    const int xp = j & 1;
    const uint32_t xph = (uint32_t)(j >> 1) & 1u;
    const float* st = tile + (j % STAGES) * stage_floats;
    // the next item's row scales and prior masses: loaded now, used from its forward part on
    const int item_n = item + G;
    const bool has_next = item_n < n_items;
    const float den_n = has_next ? den_prefetch(den, item_n / nmb, T, cta_t0 - 1, R) : 0.f;
    const float2 w_n = has_next ? load_w(item_n) : make_float2(0.f, 0.f);
    const float* s_dqf = st + o;
    const float* s_dk = st + TILE + o;
    const float* s_k = st + 2 * TILE + 32 + o;  // k_t = r_{t-1}
    const float* s_r = st + 2 * TILE + 64 + o;  // r_t
    const float* s_dqo = st + 3 * TILE + 64 + o;
    const float* si = sinv[j & 1] + rh;  // si[i]: scale of k row i, si[i + 1]: of r row i
    const float2 wm = w_cur;

    // carry of the forward scan into this thread's rows: lower ranks' totals, lower warps', then
    // (second half) the first half's
    if (cr > 0 && !mbar_wait_bounded(&xbar_f[xp], xph, ok_flag ? 2000000000ull : SCAN_SHORT_WAIT_NS)) {
      raise_device_error(DEVERR_SCAN_TMA_WAIT);
      ok_flag = 0;
    }
    float2 n = make_float2(0.f, 0.f);
#pragma unroll
    for (int jj = 0; jj < SCAN_MAX_CLUSTER; ++jj)
      if (jj < cr) {
        const float2 t2 = *reinterpret_cast<const float2*>(&ctot_f[xp][jj][s2]);
        n.x = fmaf(n.x, lam_cta, t2.x);
        n.y = fmaf(n.y, lam_cta, t2.y);
      }
#pragma unroll
    for (int jj = 0; jj < WARPS; ++jj)
      if (jj < wp) {
        const float2 t2 = *reinterpret_cast<const float2*>(&warp_sum_f[xp][jj][s2]);
        n.x = fmaf(n.x, lam_seg, t2.x);
        n.y = fmaf(n.y, lam_seg, t2.y);
      }
    if (half) {
      n.x = fmaf(lam_h, n.x, lo_cur.x);
      n.y = fmaf(lam_h, n.y, lo_cur.y);
    }

    float2 dw_acc = make_float2(0.f, 0.f);
    float dg_f = 0.f;
    float2 drd_v[H], dc_v[H];
#pragma unroll
    for (int i = 0; i < H; ++i) {
      const int t = t0 + i;
      const bool live = t < T && valid;
      const float2 k2 = *reinterpret_cast<const float2*>(s_k + i * 32);
      const float2 r2 = *reinterpret_cast<const float2*>(s_r + i * 32);
      const float2 dqfv = *reinterpret_cast<const float2*>(s_dqf + i * 32);
      const float2 dqov = has_dqo ? *reinterpret_cast<const float2*>(s_dqo + i * 32) : make_float2(0.f, 0.f);
      const float sk = si[i], sr = si[i + 1];
      n.x = fmaf(lam, n.x, k2.x * sk);
      n.y = fmaf(lam, n.y, k2.y * sk);
      float cx = wm.x + n.x, cy = wm.y + n.y;
      float ix = fast_rcp(cx), iy = fast_rcp(cy);
      float qx = (r2.x * sr) * ix, qy = (r2.y * sr) * iy;
      if (!live) {
        cx = cy = 1.f;
        qx = qy = 0.f;
        ix = iy = 1.f;
      }
      const float drx = (dqfv.x + dqov.x) * ix, dry = (dqfv.y + dqov.y) * iy;
      const float dcx = -drx * qx, dcy = -dry * qy;
      drd_v[i] = make_float2(drx, dry);
      dc_v[i] = make_float2(dcx, dcy);
      dw_acc.x += dcx;
      dw_acc.y += dcy;
      float tx = dcx * (cx - wm.x), ty = dcy * (cy - wm.y);
      if (fast_identity) {
        tx += qx * dqfv.x;
        ty += qy * dqfv.y;
      }
      dg_f = fmaf((float)t - t_mid, tx, dg_f);
      dg_f = fmaf((float)t - t_mid, ty, dg_f);
    }
    // this thread's reverse sum over its rows; the warp's = the first half's + lam^H x the second's
    float2 run = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = H - 1; i >= 0; --i) {
      run.x = fmaf(lam, run.x, dc_v[i].x);
      run.y = fmaf(lam, run.y, dc_v[i].y);
    }
    const int up = (lane & 15) + 16;
    const float2 hi = make_float2(__shfl_sync(0xffffffffu, run.x, up), __shfl_sync(0xffffffffu, run.y, up));
    const float2 dw_hi = make_float2(__shfl_sync(0xffffffffu, dw_acc.x, up), __shfl_sync(0xffffffffu, dw_acc.y, up));
    if (!half) {
      *reinterpret_cast<float2*>(&warp_sum[wp][s2]) = make_float2(fmaf(lam_h, hi.x, run.x), fmaf(lam_h, hi.y, run.y));
      *reinterpret_cast<float2*>(&warp_dw[wp][s2]) = make_float2(dw_acc.x + dw_hi.x, dw_acc.y + dw_hi.y);
    }
    __syncthreads();
    // every thread is past the wait on xbar_f[xp]: armed for item j + 2, whose forward totals the
    // lower ranks send only after this CTA's reverse totals of item j (below) have reached them
    if (threadIdx.x == 0 && cr > 0) mbar_arrive_expect_tx(&xbar_f[xp], (uint32_t)cr * 128u);
    if (wp == 0) {
      float tot = 0.f;
      for (int jj = WARPS - 1; jj >= 0; --jj) tot = fmaf(tot, lam_seg, warp_sum[jj][lane]);
      const uint32_t slot = smem_u32(&ctot_r[xp][cr][lane]), xb = smem_u32(&xbar_r[xp]);
      for (int jj = 0; jj < cr; ++jj) st_async_f32(mapa_shared(slot, jj), tot, mapa_shared(xb, jj));
      const int ml = (item % nmb) * 32 + lane;
      if (ml < M) {
        float sdw = 0.f;
        for (int jj = 0; jj < WARPS; ++jj) sdw += warp_dw[jj][lane];
        part_dw[((int64_t)b * C + cr) * M + ml] = sdw;
      }
    }
    float2 lo_n = make_float2(0.f, 0.f);
    if (has_next) {
      den_store(sinv[(j + 1) & 1], den, den_n, T, cta_t0 - 1, R);  // last read in item j - 1
      lo_n = forward_part(j + 1);
    }
    if (cr < C - 1 && !mbar_wait_bounded(&xbar_r[xp], xph, ok_flag ? 2000000000ull : SCAN_SHORT_WAIT_NS)) {
      raise_device_error(DEVERR_SCAN_TMA_WAIT);
      ok_flag = 0;
    }
    // dkc just past this thread's rows: higher ranks' totals, higher warps', then (first half) the
    // second half's
    float2 carry = make_float2(0.f, 0.f);
#pragma unroll
    for (int jj = SCAN_MAX_CLUSTER - 1; jj >= 0; --jj)
      if (jj < C && jj > cr) {
        const float2 t2 = *reinterpret_cast<const float2*>(&ctot_r[xp][jj][s2]);
        carry.x = fmaf(carry.x, lam_cta, t2.x);
        carry.y = fmaf(carry.y, lam_cta, t2.y);
      }
#pragma unroll
    for (int jj = WARPS - 1; jj >= 0; --jj)
      if (jj > wp) {
        const float2 t2 = *reinterpret_cast<const float2*>(&warp_sum[jj][s2]);
        carry.x = fmaf(carry.x, lam_seg, t2.x);
        carry.y = fmaf(carry.y, lam_seg, t2.y);
      }
    if (!half) {
      carry.x = fmaf(lam_h, carry.x, hi.x);
      carry.y = fmaf(lam_h, carry.y, hi.y);
    }
    dg_acc += (double)dg_f;
    if (valid) {
      const int64_t base = (int64_t)b * T * M + m0;
      const int t_end = t0 + H;
      float2 dkt_next = make_float2(0.f, 0.f);  // dk_total of the row after this thread's last one
      if (t_end < T) {
        const float2 d2 = *reinterpret_cast<const float2*>(s_dk + H * 32);  // the dk tile holds row t_end
        dkt_next = make_float2(d2.x + carry.x, d2.y + carry.y);
      }
      run = carry;
      float dg_s = 0.f;
#pragma unroll
      for (int i = H - 1; i >= 0; --i) {
        const int t = t0 + i;
        if (t < T) {
          const float2 dkv = *reinterpret_cast<const float2*>(s_dk + i * 32);
          const float2 k2 = *reinterpret_cast<const float2*>(s_k + i * 32);
          const float kx = k2.x * si[i], ky = k2.y * si[i];
          run.x = fmaf(lam, run.x, dc_v[i].x);  // dkc_t
          run.y = fmaf(lam, run.y, dc_v[i].y);
          *reinterpret_cast<float2*>(dr + base + (int64_t)t * M) =
              make_float2(drd_v[i].x + dkt_next.x, drd_v[i].y + dkt_next.y);
          dkt_next = make_float2(dkv.x + run.x, dkv.y + run.y);
          float tx = -kx * run.x, ty = -ky * run.y;
          if (fast_identity) {
            tx -= kx * dkv.x;
            ty -= ky * dkv.y;
          }
          dg_s = fmaf((float)t - t_mid, tx, dg_s);
          dg_s = fmaf((float)t - t_mid, ty, dg_s);
        }
      }
      dg_acc += (double)dg_s;
    }
    w_cur = w_n;
    lo_cur = lo_n;
    __syncthreads();  // this item's stage, sinv[j & 1], warp_sum and warp_dw are free again
    if (threadIdx.x == 0) {
      if (cr < C - 1) mbar_arrive_expect_tx(&xbar_r[xp], (uint32_t)(C - 1 - cr) * 128u);
      fence_proxy_async_smem();
      issue(j + STAGES);
    }
  }
  red_dg[threadIdx.x] = dg_acc;
  __syncthreads();
  for (int stride = 16 * WARPS; stride > 0; stride >>= 1) {
    if ((int)threadIdx.x < stride) red_dg[threadIdx.x] += red_dg[threadIdx.x + stride];
    __syncthreads();
  }
  if (threadIdx.x == 0) part_dg[blockIdx.x] = red_dg[0];
  // no CTA leaves while a peer may still send into its shared memory
  __syncwarp();
  cluster_sync_all();
}

// 3-D map over an fp32 (B, T, M) array with a 32-slot x `rows` box, no swizzle.
inline int make_rows_tmap(CUtensorMap* map, const float* ptr, int64_t B, int64_t T, int64_t M, int rows) {
  auto fn = encode_tiled();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return ULM_ERR_UNSUPPORTED;
  }
  cuuint64_t dims[3] = {(cuuint64_t)M, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)M * 4, (cuuint64_t)(T * M) * 4};
  cuuint32_t box[3] = {32, (cuuint32_t)rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (scan tile) failed (%d)", (int)r);
    return ULM_ERR_CUDA;
  }
  return ULM_OK;
}

// TMA-staged scans need 16-byte aligned bases and rows (M % 4 == 0) and T <= 8 * 256.
struct TmaScanPlan {
  int seg, warps, ctas;
};

inline TmaScanPlan plan_tma_scan(int64_t T, int64_t M, const void* const* ptrs, int n) {
  if (M % 4 != 0) return {0, 0, 0};
  for (int i = 0; i < n; ++i)
    if (ptrs[i] && !is_aligned16(ptrs[i])) return {0, 0, 0};
  if (T <= 8 * 128) return {16, 8, (int)cdiv(T, 128)};
  if (T <= 8 * 256) return {16, 16, (int)cdiv(T, 256)};
  return {0, 0, 0};
}

template <typename K, typename... Args>
int launch_cluster_smem(K kernel, dim3 grid, int threads, int cluster_x, size_t smem, cudaStream_t st,
                        Args... args) {
  ULM_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled();
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  ULM_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, args...));
  return ULM_OK;
}

// library-wide choice of scan kernels (ulm_set_scan_mode): 1 = persistent pipelined, 0 = per item
static int g_scan_mode = 1;
constexpr int SCAN_PIPE_STAGES = 2;  // backward: two stages of up to 66 KB
constexpr int SCAN_FWD_STAGES = 2;   // forward: two stages of 16.5 KB (more CTAs per SM beat a deeper ring)

// Ticket pairs (next ticket, clusters done) of the forward scan's item dealing, per device. Each
// launch takes the next pair of the ring; the last cluster of a launch resets its pair, so a pair
// is reused only SCAN_TICKET_PAIRS launches later, long after the launch that used it has ended.
constexpr int SCAN_TICKET_PAIRS = 4096;
__device__ unsigned int g_scan_tickets[SCAN_TICKET_PAIRS][2];

// The pair for the next launch on stream st; NULL (fixed items) while st is being captured into a
// graph, which may be replayed on several streams at once.
unsigned int* scan_tickets(cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (cs != cudaStreamCaptureStatusNone) return nullptr;
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return nullptr;
  static std::mutex mu;
  static unsigned int* base[64] = {};
  static unsigned int next[64] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (!base[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_scan_tickets) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    base[dev] = static_cast<unsigned int*>(p);
  }
  const unsigned int k = next[dev]++ % SCAN_TICKET_PAIRS;
  return base[dev] + 2 * k;
}

// Clusters of a persistent scan that fit on the device at once (cached per device, kernel and
// shared-memory size), at most n_items.
template <typename K>
int pipe_clusters(K kernel, int threads, int C, size_t smem, int64_t n_items, int* out) {
  struct Entry {
    int dev, C;
    const void* fn;
    size_t smem;
    int n;
  };
  static std::mutex mu;
  static Entry cache[32];
  static int n_cache = 0;
  const int dev = current_device();
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < n_cache; ++i)
      if (cache[i].dev == dev && cache[i].C == C && cache[i].fn == (const void*)kernel && cache[i].smem == smem) {
        *out = (int)std::min<int64_t>(cache[i].n, n_items);
        return ULM_OK;
      }
  }
  ULM_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  ULM_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, kernel, &cfg));
  ULM_REQUIRE(n > 0, "no cluster of %d CTAs with %zu bytes of shared memory fits on the device", C, smem);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (n_cache < 32) cache[n_cache++] = Entry{dev, C, (const void*)kernel, smem, n};
  }
  *out = (int)std::min<int64_t>(n, n_items);
  return ULM_OK;
}


// dg = sum of part_dg (n1 doubles) + sum of extra (n2 floats): one block, every thread sums a fixed
// strided subset in order, then a fixed-shape tree. Deterministic for given inputs.
__global__ void __launch_bounds__(256)
    stats_bwd_dg_kernel(const double* __restrict__ part_dg, int64_t n1, const float* __restrict__ extra, int64_t n2,
                        float* __restrict__ dg) {
  pdl_enter();
  __shared__ double red[256];
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < n1; i += 256) s += part_dg[i];
  for (int64_t i = threadIdx.x; i < n2; i += 256) s += (double)extra[i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int stride = 128; stride > 0; stride >>= 1) {
    if ((int)threadIdx.x < stride) red[threadIdx.x] += red[threadIdx.x + stride];
    __syncthreads();
  }
  if (threadIdx.x == 0) *dg = (float)red[0];
}

// scratch layout: [part_dw: B*8*M float][part_dg: B*groups double][tile partials: n float]
// (8 = largest cluster; groups = dg partials per batch row, at most 8 per 32-slot tile)
struct StatsScratch {
  float* part_dw;
  double* part_dg;
  float* tiles;
};

inline int64_t align256(int64_t n) { return (n + 255) / 256 * 256; }

inline int64_t stats_dg_groups(int64_t M) { return cdiv(M, 32) * 8; }

inline StatsScratch carve_stats_scratch(void* base, int64_t B, int64_t M) {
  const int64_t groups = stats_dg_groups(M);
  char* p = static_cast<char*>(base);
  StatsScratch s;
  s.part_dw = reinterpret_cast<float*>(p);
  p += align256(B * 8 * M * 4);
  s.part_dg = reinterpret_cast<double*>(p);
  p += align256(B * groups * 8);
  s.tiles = reinterpret_cast<float*>(p);
  return s;
}

// Can the TMA-staged scans handle this shape (and so the backward rebuild q and c)?
// Shared by the public statistics backward (fast_identity = 1, the reference's K5 semantics) and
// the operator backward (fast_identity = 0, tile partials of the score epilogue added instead).
// q == c == nullptr selects the recompute mode (TMA path only).
int stats_bwd_run(const float* dqf, const float* dq_out, const float* dk, const float* q, const float* c,
                  const float* r, const float* den, const float* w, const float* g, float* dr, float* dw, float* dg,
                  void* partial, int64_t B, int64_t T, int64_t M, int fast_identity, const float* tile_partials,
                  int64_t n_tiles, cudaStream_t st, cudaStream_t red_st) {
  StatsScratch sc = carve_stats_scratch(partial, B, M);
  int64_t n_dg, dw_rows;
  const bool recompute = q == nullptr && c == nullptr;
  const void* ptrs[7] = {dqf, dq_out, dk, q, c, r, dr};
  const TmaScanPlan tp = plan_tma_scan(T, M, ptrs, 7);
  ULM_REQUIRE((tp.ctas && tp.seg * tp.warps + 1 <= 256) || !recompute,
              "q and c may be omitted only when M %% 4 == 0, T <= 1024 and every array is 16-byte aligned");
  ULM_REQUIRE(recompute || (q && c), "q and c must both be given or both be NULL");
  if (tp.ctas) {
    const int R = tp.seg * tp.warps;
    CUtensorMap mdqf, mdqo, mq, mc, mdk, mr;
    if (int rc = make_rows_tmap(&mdqf, dqf, B, T, M, R)) return rc;
    if (int rc = make_rows_tmap(&mdqo, dq_out ? dq_out : dqf, B, T, M, R)) return rc;
    if (int rc = make_rows_tmap(&mq, recompute ? dqf : q, B, T, M, R)) return rc;
    if (int rc = make_rows_tmap(&mc, recompute ? dqf : c, B, T, M, R)) return rc;
    if (int rc = make_rows_tmap(&mdk, dk, B, T, M, R)) return rc;
    if (int rc = make_rows_tmap(&mr, r, B, T, M, recompute ? R + 1 : R)) return rc;
    const int C = tp.ctas;
    dim3 grid((unsigned)(cdiv(M, 32) * C), (unsigned)B);
    const size_t smem = (size_t)((recompute ? 3 * R + 1 : 5 * R) + (dq_out ? R : 0)) * 32 * 4;
    const int hq = dq_out ? 1 : 0;
    int rc;
    if (g_scan_mode == 1 && recompute && tp.warps == 8) {
      const int64_t n_items = B * cdiv(M, 32);
      const size_t smem_p = (size_t)(3 * R + 2 + (dq_out ? R : 0)) * 32 * 4 * SCAN_PIPE_STAGES;
      auto kern = stats_bwd_pipe_kernel<16, 8, SCAN_PIPE_STAGES>;
      CUtensorMap mdk1;
      if ((rc = make_rows_tmap(&mdk1, dk, B, T, M, R + 1))) return rc;
      int nc = 0;
      if ((rc = pipe_clusters(kern, 256, C, smem_p, n_items, &nc))) return rc;
      const dim3 pgrid((unsigned)(nc * C));
      rc = launch_cluster_smem(kern, pgrid, 256, C, smem_p, st, mdqf, mdqo, mdk1, mr, den, w, g, dr, sc.part_dw,
                               sc.part_dg, (int)B, (int)T, (int)M, hq, fast_identity);
      if (rc) return rc;
      n_dg = pgrid.x;  // one partial per CTA (at most B x cdiv(M, 32) x 8)
      dw_rows = B * C;
    } else {
#define ULM_BWD_TMA(W, RC)                                                                                       \
  rc = launch_cluster_smem(stats_bwd_tma_kernel<16, W, RC>, grid, 32 * W, C, smem, st, mdqf, mdqo, mq, mc, mdk, mr, \
                           dk, den, w, g, dr, sc.part_dw, sc.part_dg, (int)T, (int)M, hq, fast_identity)
      if (tp.warps == 8) {
        if (recompute) ULM_BWD_TMA(8, true); else ULM_BWD_TMA(8, false);
      } else {
        if (recompute) ULM_BWD_TMA(16, true); else ULM_BWD_TMA(16, false);
      }
#undef ULM_BWD_TMA
      if (rc) return rc;
      n_dg = B * (int64_t)grid.x;
      dw_rows = B * C;
    }
  } else {
    const int64_t groups = cdiv(M, 32);
    dim3 grid((unsigned)groups, (unsigned)B);
    stats_bwd_kernel<<<grid, STATS_THREADS, 0, st>>>(dqf, dq_out, dk, q, c, r, den, w, g, dr, sc.part_dw,
                                                     sc.part_dg, (int)T, (int)M, fast_identity);
    ULM_LAUNCH_CHECK("stats_bwd_kernel");
    n_dg = B * groups;
    dw_rows = B;
  }
  // the dw / dg reductions on red_st when given (forked after the scan; the caller joins)
  cudaStream_t rs = st;
  if (red_st && red_st != st) {
    if (int rc = stream_after(red_st, st)) return rc;
    rs = red_st;
  }
  // dw = the (b, rank) partial rows summed in a fixed order (a tree when there are many)
  if (int rc = ::sum_parts(static_cast<const float*>(sc.part_dw), dw_rows, M, dw, rs)) return rc;
  if (int rc = launch_pdl(stats_bwd_dg_kernel, dim3(1), dim3(256), 0, rs, (const double*)sc.part_dg, n_dg,
                          tile_partials, tile_partials ? n_tiles : (int64_t)0, dg))
    return rc;
  return ULM_OK;
}

}  // namespace ulm

using namespace ulm;

int stats_fwd_run(const float* r, const float* den, const float* w, const float* g, float* q, float* c, void* qop,
                  void* kop, int op_dtype, int64_t ld_op, int64_t B, int64_t T, int64_t M, void* stream);

extern "C" int ulm_memory_stats_fwd(const float* r, const float* w, const float* g, float* q, float* c, void* qop,
                                    void* kop, int op_dtype, int64_t ld_op, int64_t B, int64_t T, int64_t M,
                                    void* stream) {
  return stats_fwd_run(r, nullptr, w, g, q, c, qop, kop, op_dtype, ld_op, B, T, M, stream);
}

int stats_fwd_run(const float* r, const float* den, const float* w, const float* g, float* q, float* c, void* qop,
                  void* kop, int op_dtype, int64_t ld_op, int64_t B, int64_t T, int64_t M, void* stream) {
  ULM_REQUIRE(B >= 0 && T >= 0 && M >= 0, "negative extent");
  if (B == 0 || T == 0 || M == 0) return ULM_OK;
  ULM_REQUIRE(r && w && g && qop && kop, "null pointer argument");
  ULM_REQUIRE(q || !c, "q may be omitted only together with c");
  ULM_REQUIRE(ld_op >= M, "ld_op (%lld) < M (%lld)", (long long)ld_op, (long long)M);
  ULM_REQUIRE(op_dtype == ULM_F32 || op_dtype == ULM_BF16, "op_dtype must be ULM_F32 or ULM_BF16");
  ULM_REQUIRE(B <= 65535 && T < (1ll << 31) && M < (1ll << 31), "extent too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const void* ptrs[3] = {r, q, c};
  const TmaScanPlan tp = plan_tma_scan(T, M, ptrs, 3);
  ULM_REQUIRE(c || tp.ctas, "c may be omitted only when M %% 4 == 0, T <= 2048 and r, q are 16-byte aligned");
  if (tp.ctas) {
    const int R = tp.seg * tp.warps;
    CUtensorMap mr;
    CUtensorMap mr1;
    if (int rc = make_rows_tmap(&mr, r, B, T, M, R)) return rc;
    if (int rc = make_rows_tmap(&mr1, r, B, T, M, 1)) return rc;
    const int C = tp.ctas;
    dim3 grid((unsigned)(cdiv(M, 32) * C), (unsigned)B);
    const size_t smem = (size_t)(R + 1) * 32 * 4;
    const bool bf = op_dtype == ULM_BF16;
    if (g_scan_mode == 1 && tp.warps == 8) {
      const int64_t n_items = B * cdiv(M, 32);
      const size_t smem_p = smem * SCAN_FWD_STAGES;
      auto kb = stats_fwd_pipe_kernel<16, 8, SCAN_FWD_STAGES, __nv_bfloat16>;
      auto kf = stats_fwd_pipe_kernel<16, 8, SCAN_FWD_STAGES, float>;
      int nc = 0;
      if (int rc = bf ? pipe_clusters(kb, 256, C, smem_p, n_items, &nc) : pipe_clusters(kf, 256, C, smem_p, n_items, &nc))
        return rc;
      const dim3 pgrid((unsigned)(nc * C));
      unsigned int* tk = scan_tickets(st);
      return bf ? launch_cluster_smem(kb, pgrid, 256, C, smem_p, st, mr, mr1, den, w, g, q, c, qop, kop, ld_op, (int)B,
                                      (int)T, (int)M, tk)
                : launch_cluster_smem(kf, pgrid, 256, C, smem_p, st, mr, mr1, den, w, g, q, c, qop, kop, ld_op, (int)B,
                                      (int)T, (int)M, tk);
    }
    if (tp.warps == 8)
      return bf ? launch_cluster_smem(stats_fwd_tma_kernel<16, 8, __nv_bfloat16>, grid, 256, C, smem, st, mr, mr1, den, w,
                                      g, q, c, qop, kop, ld_op, (int)T, (int)M)
                : launch_cluster_smem(stats_fwd_tma_kernel<16, 8, float>, grid, 256, C, smem, st, mr, mr1, den, w, g, q, c,
                                      qop, kop, ld_op, (int)T, (int)M);
    return bf ? launch_cluster_smem(stats_fwd_tma_kernel<16, 16, __nv_bfloat16>, grid, 512, C, smem, st, mr, mr1, den, w,
                                    g, q, c, qop, kop, ld_op, (int)T, (int)M)
              : launch_cluster_smem(stats_fwd_tma_kernel<16, 16, float>, grid, 512, C, smem, st, mr, mr1, den, w, g, q, c,
                                    qop, kop, ld_op, (int)T, (int)M);
  }
  dim3 grid((unsigned)cdiv(M, 32), (unsigned)B);
  if (op_dtype == ULM_BF16)
    stats_fwd_kernel<__nv_bfloat16><<<grid, STATS_THREADS, 0, st>>>(r, den, w, g, q, c, qop, kop, ld_op, (int)T,
                                                                    (int)M);
  else
    stats_fwd_kernel<float><<<grid, STATS_THREADS, 0, st>>>(r, den, w, g, q, c, qop, kop, ld_op, (int)T, (int)M);
  ULM_LAUNCH_CHECK("stats_fwd_kernel");
  return ULM_OK;
}

extern "C" int64_t ulm_memory_stats_bwd_scratch(int64_t B, int64_t T, int64_t M) {
  if (B < 0 || T < 0 || M < 0) return -1;
  return align256(B * 8 * M * 4) + align256(B * stats_dg_groups(M) * 8) + align256(decay_dg_partials(B, T) * 4);
}

extern "C" int ulm_memory_stats_bwd(const float* dqf, const float* dq_out, const float* dk, const float* q,
                                    const float* c, const float* r, const float* w, const float* g, float* dr,
                                    float* dw, float* dg, void* partial, int64_t B, int64_t T, int64_t M,
                                    void* stream) {
  ULM_REQUIRE(B >= 0 && T >= 0 && M >= 0, "negative extent");
  ULM_REQUIRE(dg && (dw || M == 0), "null dw/dg");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B == 0 || T == 0 || M == 0) {
    if (M > 0) ULM_CUDA_TRY(cudaMemsetAsync(dw, 0, M * sizeof(float), st));
    ULM_CUDA_TRY(cudaMemsetAsync(dg, 0, sizeof(float), st));
    return ULM_OK;
  }
  ULM_REQUIRE(dqf && dk && r && w && g && dr && partial, "null pointer argument");
  ULM_REQUIRE(B <= 65535 && T < (1ll << 31) && M < (1ll << 31), "extent too large");
  return stats_bwd_run(dqf, dq_out, dk, q, c, r, nullptr, w, g, dr, dw, dg, partial, B, T, M, 1, nullptr, 0, st, nullptr);
}

// ---- statistics backward without any allocation ------------------------------------------------
// Some hosts cannot hand this library device memory at call time: a serving runtime that reserves
// all of HBM for its own pool at start-up, or a plugin host that owns every device allocation.
// For them the statistics backward can use a fixed scratch block that lives in the library's own
// device image (ULM_NOALLOC_SCRATCH_BYTES per device, held by every GPU that loads the library until
// the process exits). Host code cannot pass the array's name to a kernel (on the host it is only
// a stand-in symbol), so its device address is looked up with cudaGetSymbolAddress in the calling
// thread's current context. Outside stream capture every call looks it up again (so a context
// created later, or the primary context after cudaDeviceReset, gets its own address); during a
// capture the address recorded for the current context by an earlier call is used, and a capture
// with no earlier call in that context is refused.

static __device__ __align__(256) unsigned char g_noalloc_scratch[ULM_NOALLOC_SCRATCH_BYTES];

namespace {

std::mutex g_noalloc_mu;
constexpr int NOALLOC_CONTEXTS = 64;
CUcontext g_noalloc_ctx[NOALLOC_CONTEXTS] = {};
void* g_noalloc_addr[NOALLOC_CONTEXTS] = {};
int g_noalloc_next = 0;  // next table entry to (re)use once all are taken

// Bytes the public statistics backward actually uses (no score-epilogue partials).
int64_t stats_bwd_core_scratch(int64_t B, int64_t M) {
  return align256(B * 8 * M * 4) + align256(B * stats_dg_groups(M) * 8);
}

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

int noalloc_scratch(cudaStream_t st, void** out) {
  const int dev = current_device();
  ULM_REQUIRE(dev >= 0, "no current CUDA device");
  // a runtime call on the stream first: it makes the device's primary context current if the
  // thread has none yet
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  ULM_CUDA_TRY(cudaStreamIsCapturing(st, &cs));
  CtxGetCurrentFn get = ctx_get_current();
  ULM_REQUIRE(get, "cuCtxGetCurrent is not available from the driver");
  CUcontext ctx = nullptr;
  ULM_REQUIRE(get(&ctx) == CUDA_SUCCESS && ctx, "no current CUDA context");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  int slot = -1;
  for (int i = 0; i < NOALLOC_CONTEXTS; ++i)
    if (g_noalloc_ctx[i] == ctx) slot = i;
  if (cs != cudaStreamCaptureStatusNone) {
    ULM_REQUIRE(slot >= 0 && g_noalloc_addr[slot],
                "ulm_memory_stats_bwd_noalloc: first call in this context during stream capture; make one call "
                "outside capture first");
    *out = g_noalloc_addr[slot];
    return ULM_OK;
  }
  void* p = nullptr;
  ULM_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
  ULM_REQUIRE(p != nullptr, "cudaGetSymbolAddress returned a null scratch address");
  if (slot < 0) {
    for (int i = 0; i < NOALLOC_CONTEXTS && slot < 0; ++i)
      if (!g_noalloc_ctx[i]) slot = i;
    if (slot < 0) slot = g_noalloc_next++ % NOALLOC_CONTEXTS;
    g_noalloc_ctx[slot] = ctx;
  }
  g_noalloc_addr[slot] = p;
  *out = p;
  return ULM_OK;
}

}  // namespace

extern "C" int ulm_memory_stats_bwd_noalloc(const float* dqf, const float* dq_out, const float* dk, const float* q,
                                            const float* c, const float* r, const float* w, const float* g,
                                            float* dr, float* dw, float* dg, int64_t B, int64_t T, int64_t M,
                                            void* stream) {
  ULM_REQUIRE(B >= 0 && T >= 0 && M >= 0, "negative extent");
  ULM_REQUIRE(dg && (dw || M == 0), "null dw/dg");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B == 0 || T == 0 || M == 0) {
    // the same result as ulm_memory_stats_bwd for empty extents: dw and dg are zero
    if (M > 0) ULM_CUDA_TRY(cudaMemsetAsync(dw, 0, M * sizeof(float), st));
    ULM_CUDA_TRY(cudaMemsetAsync(dg, 0, sizeof(float), st));
    return ULM_OK;
  }
  ULM_REQUIRE(dqf && dk && r && w && g && dr, "null pointer argument");
  ULM_REQUIRE(B <= 65535 && T < (1ll << 31) && M < (1ll << 31), "extent too large");
  const int64_t need = stats_bwd_core_scratch(B, M);
  ULM_REQUIRE(need <= (int64_t)ULM_NOALLOC_SCRATCH_BYTES,
              "ulm_memory_stats_bwd_noalloc: B=%lld x M=%lld needs %lld bytes of scratch, the built-in block holds "
              "%lld; use ulm_memory_stats_bwd with caller-provided scratch",
              (long long)B, (long long)M, (long long)need, (long long)ULM_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(st, &scratch)) return rc;
  // every scratch entry the kernels read is written earlier in the same call: nothing to clear
  return stats_bwd_run(dqf, dq_out, dk, q, c, r, nullptr, w, g, dr, dw, dg, scratch, B, T, M, 1, nullptr, 0, st, nullptr);
}

extern "C" int ulm_set_scan_mode(int mode) {
  if (mode < 0 || mode > 1) return -1;
  const int old = g_scan_mode;
  g_scan_mode = mode;
  return old;
}

extern "C" int ulm_memory_needs_c(int64_t T, int64_t M) {
  // whether the operator backward needs the saved c: it rebuilds q and c on the TMA scan path when
  // one CTA's r tile plus one row fits a TMA box (M % 4 == 0, T <= 1024; buffers 16-byte aligned)
  const void* none[1] = {nullptr};
  const TmaScanPlan tp = plan_tma_scan(T, M, none, 0);
  return (tp.ctas && tp.seg * tp.warps + 1 <= 256) ? 0 : 1;
}
