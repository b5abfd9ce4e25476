// The two back ends of the batched GEMM engine (see gemm.cuh).
//
// Tensor-core back end (bf16 operands): persistent, warp-specialised sm_100a kernels, on single
// CTAs (tc_gemm_kernel: 128 x BN tiles) or on CTA pairs (tc2_gemm_kernel: 256 x 256 tiles,
// cta_group::2, each CTA holding 128 rows of A and 128 columns of B).
//   warp 0        : TMA producer - 128B-swizzled tiles of A and B (64 k values) per stage
//   warp 1        : allocates TMEM, one elected lane (of the pair's leader CTA) issues tcgen05.mma
//                   (K=16 steps) into a double-buffered fp32 accumulator (2 x BN TMEM columns)
//   warps 2..9    : epilogue - EPI_WARPS = 8 warps, two per TMEM lane quadrant, each with half of
//                   the tile's columns: tcgen05.ld 16 columns at a time, the fused epilogue
//                   arithmetic, two 4 KB swizzled shared-memory staging tiles per warp and TMA
//                   tensor stores (tile aux operands arrive the same way, loaded ahead)
// Stage hand-offs use mbarriers; the accumulator is double-buffered so the epilogue of tile i
// overlaps the MMAs of tile i+1. Every wait is bounded: on timeout the kernel records a device
// error, drains what it has in flight, frees its TMEM and returns.
//
// FMA back end (fp32 operands): 64 x 64 tiles, 16-deep k slices in shared memory, 4 x 4 outputs
// per thread, same tile decomposition and epilogue semantics.
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "gemm.cuh"

namespace ulm {

// ------------------------------------------------------------------------------------------------
// epilogue: one thread owns one output row segment of 32 columns

__host__ __device__ __forceinline__ bool has_tile_aux(int kind) { return kind == EPI_DECAY_DG || kind == EPI_STORE_ADD; }

// NC consecutive elements of an aux row (EPI_DECAY_DG: the forward's scores; EPI_STORE_ADD: the
// fp32 addend; both in the output's type) as floats; zero past `ncols`.
template <int NC>
__device__ __forceinline__ void load_aux(const GemmEpilogue& e, int b, int row, int col0, int ncols, float (&p)[NC]) {
  const int64_t off = (int64_t)b * e.aux_bstride + (int64_t)row * e.ld_aux + col0;
  if (e.out_dtype == ULM_F32) {
    const float* a = reinterpret_cast<const float*>(e.aux) + off;
    if (ncols == NC && e.vec_ok) {
#pragma unroll
      for (int i = 0; i < NC; i += 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(a + i);
        p[i] = a4.x;
        p[i + 1] = a4.y;
        p[i + 2] = a4.z;
        p[i + 3] = a4.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < NC; ++i) p[i] = i < ncols ? a[i] : 0.f;
    }
  } else {
    const __nv_bfloat16* a = reinterpret_cast<const __nv_bfloat16*>(e.aux) + off;
    if (ncols == NC && e.vec_ok) {
#pragma unroll
      for (int i = 0; i < NC; i += 8) {
        const uint4 pk = *reinterpret_cast<const uint4*>(a + i);
        const uint32_t w4[4] = {pk.x, pk.y, pk.z, pk.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          __nv_bfloat162 h;
          memcpy(&h, &w4[j], 4);
          const float2 f = __bfloat1622float2(h);
          p[i + 2 * j] = f.x;
          p[i + 2 * j + 1] = f.y;
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < NC; ++i) p[i] = i < ncols ? __bfloat162float(a[i]) : 0.f;
    }
  }
}

// The epilogue's arithmetic on NC accumulator values v of row `row`, columns col0..col0+NC-1
// (ncols of them inside the output); p holds the tile aux values of the same positions.
template <int NC>
__device__ __forceinline__ void epilogue_math(const GemmEpilogue& e, float gl2, int row, int col0, int ncols,
                                              float* v, const float* p, float& dg_acc) {
  if (e.kind == EPI_DECAY || e.kind == EPI_DECAY_DG) {
    // element i has lag = row - col0 - i (exact in float); decay lam^lag = 2^(gl2 lag) on and below
    // the diagonal, 0 above it
    const float lag0 = (float)(row - col0);
    if (e.kind == EPI_DECAY_DG) {
      // d/dg share: sum of lag * P * dP (P, the aux, is zero above the diagonal; lag is zero on it)
#pragma unroll
      for (int i = 0; i < NC; ++i) dg_acc = fmaf((lag0 - (float)i) * p[i], v[i], dg_acc);
    }
    if (row - col0 >= NC - 1) {
      // the whole chunk is on or below the diagonal: for i = NC-1-8j-k the factor is
      // lam^(lag0-NC+1) * lam^(8j) * lam^k, all factors <= 1, three exp2 per chunk
      static_assert(NC % 8 == 0, "chunks of 8 columns");
      const float l1 = fast_exp2(gl2);
      float pw[8];
      pw[0] = 1.f;
#pragma unroll
      for (int k = 1; k < 8; ++k) pw[k] = pw[k - 1] * l1;
      const float l8 = fast_exp2(gl2 * 8.f);
      float fj = fast_exp2(gl2 * (lag0 - (float)(NC - 1)));
#pragma unroll
      for (int j = 0; j < NC / 8; ++j) {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[NC - 1 - 8 * j - k] *= fj * pw[k];
        fj *= l8;
      }
    } else {
#pragma unroll
      for (int i = 0; i < NC; ++i) {
        const float lag = lag0 - (float)i;
        v[i] = lag >= 0.f ? v[i] * fast_exp2(gl2 * lag) : 0.f;
      }
    }
  }
  if (e.kind == EPI_RELU2) {
    const float* bias = reinterpret_cast<const float*>(e.aux) + col0;
    float bv[NC];
    if (ncols == NC && (reinterpret_cast<uintptr_t>(bias) & 15) == 0) {
#pragma unroll
      for (int i = 0; i < NC; i += 4) {
        const float4 b4 = __ldg(reinterpret_cast<const float4*>(bias + i));
        bv[i] = b4.x;
        bv[i + 1] = b4.y;
        bv[i + 2] = b4.z;
        bv[i + 3] = b4.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < NC; ++i) bv[i] = i < ncols ? bias[i] : 0.f;
    }
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const float a = v[i] + bv[i];
      v[i] = a > 0.f && i < ncols ? a * a : 0.f;
      dg_acc += v[i];  // row sum of this tile row (used when e.row_partial is set)
    }
  }
  if (e.kind == EPI_ROW_DECAY) {
    // one factor per row: lam^(rd_a + rd_s * row), all powers >= 0
    const float f = fast_exp2(gl2 * (e.rd_a + e.rd_s * (float)row));
#pragma unroll
    for (int i = 0; i < NC; ++i) v[i] *= f;
  }
  if (e.kind == EPI_STORE_ADD) {
#pragma unroll
    for (int i = 0; i < NC; ++i) v[i] += p[i];
  }
  if (e.kind == EPI_CE_GRAD) {
    const bool rv = row < e.rows_valid;
    const int64_t tgt = rv ? e.targets[row] : -1;
    const float lse = rv ? e.row_lse[row] : 0.f;
    const float sc = tgt >= 0 ? *e.scale : 0.f;
#pragma unroll
    for (int i = 0; i < NC; ++i) v[i] = (__expf(v[i] - lse) - ((int64_t)(col0 + i) == tgt ? 1.f : 0.f)) * sc;
  }
}

// EPI_LSE over NC logits of row `row` at col0 (ncols valid): merge into the running (m, s) of the
// row and record the target's logit
template <int NC>
__device__ __forceinline__ void lse_update(const GemmEpilogue& e, int row, int col0, int ncols, const float (&v)[NC],
                                             float& m, float& s) {
  if (row >= e.rows_valid || ncols <= 0) return;
  float lm = -INFINITY;
#pragma unroll
  for (int i = 0; i < NC; ++i)
    if (i < ncols) lm = fmaxf(lm, v[i]);
  const float nm = fmaxf(m, lm);
  float acc = s * __expf(m - nm);
#pragma unroll
  for (int i = 0; i < NC; ++i)
    if (i < ncols) acc += __expf(v[i] - nm);
  m = nm;
  s = acc;
  const int64_t tgt = e.targets[row];
  if (tgt >= col0 && tgt < col0 + ncols) {
#pragma unroll
    for (int i = 0; i < NC; ++i)
      if ((int64_t)(col0 + i) == tgt) e.tile_partial[row] = v[i];
  }
}

// Direct epilogue: each thread stores its own row segment (used when the output or aux layout does
// not allow the tensor-map path below).
template <int NC>
__device__ __forceinline__ void epilogue_store(const GemmEpilogue& e, const GemmShape& s, float gl2, int b, int row,
                                               int col0, float (&v)[NC], float& dg_acc) {
  if (row >= s.M || col0 >= s.N) return;
  const int ncols = min(NC, s.N - col0);
  float p[NC];
  if (has_tile_aux(e.kind)) {
    load_aux<NC>(e, b, row, col0, ncols, p);
  } else {
#pragma unroll
    for (int i = 0; i < NC; ++i) p[i] = 0.f;
  }
  epilogue_math<NC>(e, gl2, row, col0, ncols, v, p, dg_acc);
  const int64_t off = (int64_t)b * e.out_bstride + (int64_t)row * e.ldo + col0;
  if (e.out_dtype == ULM_F32) {
    float* o = reinterpret_cast<float*>(e.out) + off;
    if (ncols == NC && e.vec_ok) {
#pragma unroll
      for (int i = 0; i < NC; i += 4) *reinterpret_cast<float4*>(o + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < NC; ++i)
        if (i < ncols) o[i] = v[i];
    }
  } else {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(e.out) + off;
    if (ncols == NC && e.vec_ok) {
#pragma unroll
      for (int i = 0; i < NC; i += 8) {
        uint4 pk;
        __nv_bfloat162 p0 = __floats2bfloat162_rn(v[i], v[i + 1]);
        __nv_bfloat162 p1 = __floats2bfloat162_rn(v[i + 2], v[i + 3]);
        __nv_bfloat162 p2 = __floats2bfloat162_rn(v[i + 4], v[i + 5]);
        __nv_bfloat162 p3 = __floats2bfloat162_rn(v[i + 6], v[i + 7]);
        memcpy(&pk.x, &p0, 4);
        memcpy(&pk.y, &p1, 4);
        memcpy(&pk.z, &p2, 4);
        memcpy(&pk.w, &p3, 4);
        *reinterpret_cast<uint4*>(o + i) = pk;
      }
    } else {
#pragma unroll
      for (int i = 0; i < NC; ++i)
        if (i < ncols) o[i] = __float2bfloat16_rn(v[i]);
    }
  }
}

// Wait on an mbarrier phase unless the CTA is aborting; false on timeout or abort.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 63u) == 0u) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > 2000000000ull) {
        raise_device_error(site);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// The tile that slot t of a persistent launch with P CTAs (or CTA pairs) works on, or -1. CTA p
// takes slots p, p + P, p + 2P, ... When balanced (causal k-range products with few tiles per CTA,
// where the uneven k ranges would leave CTAs idle at the end) the tile index space is ordered by
// decreasing work (decode_tile) and every other round of P slots runs backwards (snake order),
// close to a longest-first greedy assignment; otherwise tiles are taken in index order.
__device__ __forceinline__ int schedule_tile(int t, int P, int total, int balanced) {
  if (!balanced) return t < total ? t : -1;
  const int rnd = t / P, pos = t - rnd * P;
  const int s = rnd * P + ((rnd & 1) ? P - 1 - pos : pos);
  return s < total ? s : -1;
}

// ---- staged epilogues -------------------------------------------------------------------------
// The output leaves through shared memory and TMA tensor stores, so global writes are whole lines
// instead of 32 row fragments per store instruction; a tile aux (scores / addend) arrives the same
// way through a TMA load into the staging tile, and the epilogue computes in place. Each epilogue
// warp stages 32 rows x 128 bytes (32 fp32 / 64 bf16 columns, 128-byte swizzle: one row per lane,
// conflict-free 16-byte shared stores) in two 4 KB slots of its own (EPI_MODE_WARP);
// EPI_MODE_DIRECT stores row segments straight from registers.
enum { EPI_MODE_DIRECT = 0, EPI_MODE_WARP = 1 };
// Epilogue warps per CTA: EPI_WARPS / 4 per TMEM lane quadrant, each taking an equal share (at least
// 64 columns) of the tile's columns, with SLOTS staging tiles of 4 KB (a kernel parameter: more
// slots let more aux tiles load ahead, fewer leave room for more operand stages).
constexpr int EPI_WARPS = 8;
constexpr int EPI_MAX_SLOTS = 2;
__host__ __device__ constexpr uint32_t epi_smem_bytes(int slots) { return EPI_WARPS * slots * 4096u; }

__device__ __forceinline__ uint32_t sw128_off(int r, int k) { return (uint32_t)(r * 128 + ((k ^ (r & 7)) << 4)); }

// NV values of row r of a tile with 128-byte rows (128-byte swizzle), starting at 16-byte unit u0
// (NV / 4 units in fp32, NV / 8 in bf16)
template <bool F32, int NV>
__device__ __forceinline__ void stage_write(uint8_t* tile, int r, int u0, const float* v) {
#pragma unroll
  for (int k = 0; k < (F32 ? NV / 4 : NV / 8); ++k) {
    const uint32_t off = sw128_off(r, u0 + k);
    if (F32) {
      *reinterpret_cast<float4*>(tile + off) = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
    } else {
      uint4 pk;
      __nv_bfloat162 p0 = __floats2bfloat162_rn(v[8 * k], v[8 * k + 1]);
      __nv_bfloat162 p1 = __floats2bfloat162_rn(v[8 * k + 2], v[8 * k + 3]);
      __nv_bfloat162 p2 = __floats2bfloat162_rn(v[8 * k + 4], v[8 * k + 5]);
      __nv_bfloat162 p3 = __floats2bfloat162_rn(v[8 * k + 6], v[8 * k + 7]);
      memcpy(&pk.x, &p0, 4);
      memcpy(&pk.y, &p1, 4);
      memcpy(&pk.z, &p2, 4);
      memcpy(&pk.w, &p3, 4);
      *reinterpret_cast<uint4*>(tile + off) = pk;
    }
  }
}

template <bool F32, int NV>
__device__ __forceinline__ void stage_read(const uint8_t* tile, int r, int u0, float* p) {
#pragma unroll
  for (int k = 0; k < (F32 ? NV / 4 : NV / 8); ++k) {
    const uint32_t off = sw128_off(r, u0 + k);
    if (F32) {
      const float4 a = *reinterpret_cast<const float4*>(tile + off);
      p[4 * k] = a.x;
      p[4 * k + 1] = a.y;
      p[4 * k + 2] = a.z;
      p[4 * k + 3] = a.w;
    } else {
      const uint4 pk = *reinterpret_cast<const uint4*>(tile + off);
      const uint32_t w4[4] = {pk.x, pk.y, pk.z, pk.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 h;
        memcpy(&h, &w4[j], 4);
        const float2 f = __bfloat1622float2(h);
        p[8 * k + 2 * j] = f.x;
        p[8 * k + 2 * j + 1] = f.y;
      }
    }
  }
}

// EPI_MODE_WARP: one chunk (32 rows x 128 bytes: 32 fp32 / 64 bf16 columns at col0) of the warp's
// rows row_base..+31; taddr = this warp's TMEM quadrant at the chunk's first column. n counts the
// warp's staged chunks (slot n % 2, barrier phase n / 2). False if the aux wait gave up.
// Aux tile of one staged chunk (32 rows x 128 bytes) into slot n % SLOTS of this warp; lane 0 only.
// The caller has made sure the slot's previous store has read it.
template <int SLOTS>
__device__ __forceinline__ void epi_aux_issue(const CUtensorMap* tma_aux, uint8_t* slots, uint64_t* abar, int n,
                                              int col0, int row_base, int b) {
  const int sl = n % SLOTS;
  mbar_arrive_expect_tx(&abar[sl], 4096u);
  tma_load_3d(tma_aux, slots + sl * 4096, &abar[sl], col0, row_base, b);
}

// One staged chunk of a warp: 32 rows x (32 fp32 | 64 bf16) columns through slot n % SLOTS. With a
// tile aux, the chunk's aux was issued earlier (epi_aux_issue with the same n); after the chunk's
// store the slot is refilled with the aux of the chunk SLOTS ahead (next_col0 >= 0), which then loads
// while the chunks in between are processed.
template <bool F32, int SLOTS>
__device__ __forceinline__ bool epi_chunk_warp(const GemmEpilogue& e, const GemmShape& s, const CUtensorMap* tma_out,
                                               const CUtensorMap* tma_aux, uint8_t* slots, uint64_t* abar, int& n,
                                               int& n_issued, float gl2, int b, int row_base, int col0,
                                               int next_col0, uint32_t taddr, float& dg_acc,
                                               volatile int* abort_flag, int site) {
  const int lane = threadIdx.x & 31;
  const bool aux = has_tile_aux(e.kind);
  const int sl = n % SLOTS;
  const uint32_t parity = (uint32_t)(n / SLOTS) & 1u;
  ++n;
  uint8_t* tile = slots + sl * 4096;
  if (!aux) {
    if (lane == 0) bulk_wait_group_read<SLOTS - 1>();  // the store of chunk n - SLOTS has read the slot
    __syncwarp();
  } else if (!wait_or_abort(&abar[sl], parity, abort_flag, site)) {
    return false;
  }
  // 16 columns at a time (registers: 16 accumulator + 16 aux values)
#pragma unroll 1
  for (int h = 0; h < (F32 ? 2 : 4); ++h) {
    float v[16], p[16];
    tmem_ld_32x16(taddr + (uint32_t)(16 * h), v);
    const int u0 = F32 ? 4 * h : 2 * h;
    if (aux) {
      stage_read<F32, 16>(tile, lane, u0, p);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) p[i] = 0.f;
    }
    const int c = col0 + 16 * h;
    epilogue_math<16>(e, gl2, row_base + lane, c, min(16, s.N - c), v, p, dg_acc);
    stage_write<F32, 16>(tile, lane, u0, v);
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_3d(tma_out, tile, col0, row_base, b);
    bulk_commit_group();
    if (aux && next_col0 >= 0) {
      bulk_wait_group_read<0>();  // the store just issued has read the slot
      epi_aux_issue<SLOTS>(tma_aux, slots, abar, n - 1 + SLOTS, next_col0, row_base, b);
      ++n_issued;
    }
  }
  return true;
}

// The epilogue warps (2 .. 2 + EPI_WARPS - 1) of both tensor-core kernels: for every tile of this
// CTA (t_first, t_first + t_stride, ...) wait for its accumulator, write it through the epilogue
// and hand the TMEM buffer back. Warp w reads TMEM lane quadrant w % 4 and the PART columns from
// part * PART, part = (w - 2) / 4 (warps past the tile width only keep the barrier count).
// cta_rows = the CTA's row offset inside a BM-row tile (its 128 rows); partials for EPI_DECAY_DG go
// to tile_partial[part_stride * t + part_off + (w - 2)], row sums for EPI_RELU2 and the (max, sum)
// pairs of EPI_LSE to the 64-column slot of the warp's first column.
template <int BM, int BN, bool PAIR, int SLOTS>
__device__ __forceinline__ void epilogue_warps(const GemmShape& shape, const GemmEpilogue& epi,
                                               const CUtensorMap* tma_out, const CUtensorMap* tma_aux,
                                               int m_blocks, int n_blocks, int tiles_per_batch, int total_tiles,
                                               int t_first, int t_stride, int cta_rows, uint32_t tmem_base,
                                               uint64_t* tfull, uint64_t* tempty, uint32_t leader_tempty,
                                               uint8_t* stage, uint64_t* aux_bar, volatile int* abort_flag,
                                               int site, int part_stride, int part_off) {
  constexpr int PART = BN / (EPI_WARPS / 4) < 64 ? 64 : BN / (EPI_WARPS / 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ew = warp - 2;
  const int quad = warp & 3;
  const int part = ew >> 2;
  const bool active = part * PART < BN;
  const int mode = epi.staged;
  const bool f32 = epi.out_dtype == ULM_F32;
  const float gl2 = (epi.kind == EPI_DECAY || epi.kind == EPI_DECAY_DG || epi.kind == EPI_ROW_DECAY)
                        ? (*epi.g) * 1.4426950408889634f
                        : 0.f;
  uint8_t* wslots = stage + ew * (SLOTS * 4096);  // this warp's staging tiles
  uint64_t* wbar = aux_bar + ew * SLOTS;
  int n = 0;         // staged chunks of this warp so far (slot n % SLOTS)
  int n_issued = 0;  // aux loads issued by this warp (lane 0's count)
  int j = 0;
  bool ok = true;
  const bool warp_aux = mode == EPI_MODE_WARP && has_tile_aux(epi.kind);
  const int cw = f32 ? 32 : 64;  // columns of a staged chunk
  const int rounded = (total_tiles + t_stride - 1) / t_stride * t_stride;
  for (int tt = t_first; tt < rounded; tt += t_stride) {
    const int t = schedule_tile(tt, t_stride, total_tiles, shape.balanced);
    if (t < 0) continue;
    const TileCoord tc = decode_tile<BM, BN>(t, shape, m_blocks, n_blocks, tiles_per_batch);
    const int jj = j++;
    const int acc = jj & 1;
    const uint32_t acc_phase = (uint32_t)(jj >> 1) & 1u;
    const int row_base = tc.mb * BM + cta_rows + quad * 32;
    const int row = row_base + lane;
    const int col_base = tc.nb * BN + part * PART;
    const bool cols = active && row_base < shape.M && col_base < shape.N;
    // staged chunks of this warp in this tile; with a tile aux the first SLOTS chunks' aux tiles load
    // now, while the tile's MMAs run
    const int nch = cols ? min(PART / cw, (shape.N - col_base + cw - 1) / cw) : 0;
    if (warp_aux && lane == 0 && epi.kind != EPI_LSE) {
      bulk_wait_group_read<0>();  // every earlier store of this warp has read its slot
      for (int i = 0; i < nch && i < SLOTS; ++i) {
        epi_aux_issue<SLOTS>(tma_aux, wslots, wbar, n + i, col_base + i * cw, row_base, tc.b);
        ++n_issued;
      }
    }
    if (!wait_or_abort(&tfull[acc], acc_phase, abort_flag, site)) {
      ok = false;
      break;
    }
    tc_fence_after();
    const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN + part * PART);
    float dg_acc = 0.f;
    if (!cols) {
      // nothing of this tile for this warp: only its barrier arrival below
    } else if (epi.kind == EPI_LSE) {
      float m = -INFINITY, ssum = 0.f;
#pragma unroll 1
      for (int c = 0; c < PART; c += 16) {
        float v[16];
        tmem_ld_32x16(taddr + (uint32_t)c, v);
        lse_update<16>(epi, row, col_base + c, min(16, shape.N - (col_base + c)), v, m, ssum);
      }
      if (row < shape.M) {
        float* pp = epi.row_partial + ((int64_t)row * epi.part_ld + col_base / 64) * 2;
        pp[0] = m;
        pp[1] = ssum;
      }
    } else if (mode == EPI_MODE_WARP) {
#pragma unroll 1
      for (int i = 0; i < nch && ok; ++i) {
        const int c = i * cw;
        const int next = i + SLOTS < nch ? col_base + c + SLOTS * cw : -1;
        ok = f32 ? epi_chunk_warp<true, SLOTS>(epi, shape, tma_out, tma_aux, wslots, wbar, n, n_issued, gl2, tc.b, row_base,
                                        col_base + c, next, taddr + (uint32_t)c, dg_acc, abort_flag, site)
                 : epi_chunk_warp<false, SLOTS>(epi, shape, tma_out, tma_aux, wslots, wbar, n, n_issued, gl2, tc.b,
                                         row_base, col_base + c, next, taddr + (uint32_t)c, dg_acc, abort_flag, site);
      }
    } else {
#pragma unroll 1
      for (int c = 0; c < PART; c += 16) {
        float v[16];
        tmem_ld_32x16(taddr + (uint32_t)c, v);
        epilogue_store<16>(epi, shape, gl2, tc.b, row, col_base + c, v, dg_acc);
      }
    }
    if (!ok) break;
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      if (PAIR)
        mbar_arrive_cluster(leader_tempty + (uint32_t)(acc * sizeof(uint64_t)));
      else
        mbar_arrive(&tempty[acc]);
    }
    if (epi.kind == EPI_RELU2 && epi.row_partial && cols && row < shape.M)
      epi.row_partial[((int64_t)tc.b * shape.M + row) * epi.part_ld + col_base / 64] = dg_acc;
    if (epi.kind == EPI_DECAY_DG) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dg_acc += __shfl_xor_sync(0xffffffffu, dg_acc, o);
      if (lane == 0) epi.tile_partial[part_stride * (int64_t)t + part_off + ew] = dg_acc;
    }
  }
  if (mode == EPI_MODE_WARP && lane == 0) {
    // aux loads still in flight after an abort (the last one of each slot) land before the CTA
    // exits; stores complete
    if (!ok && warp_aux) {
      for (int k = max(0, n_issued - SLOTS); k < n_issued; ++k) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&wbar[k % SLOTS], (uint32_t)(k / SLOTS) & 1u) &&
               globaltimer_ns() - t0 < 100000000ull) {
        }
      }
    }
    bulk_wait_group<0>();
  }
}

// ---- carry products ----------------------------------------------------------------------------
// A CTA (pair) of a carry product takes its tiles (slots t_first, t_first + t_stride, ...) in
// groups of two: the chunk steps of the two tiles alternate, the first in accumulator 0 and the
// second in accumulator 1, so one tile's epilogue (state write and rescale) overlaps the other
// tile's MMAs. A last group of one tile keeps accumulator 0. f(t, chunk, acc, step, steps) is
// called for every step in that order by all three roles; false stops the walk.
template <typename F>
__device__ __forceinline__ bool carry_walk(int t_first, int t_stride, int total_tiles, const GemmShape& s, F&& f) {
  const int steps = carry_steps(s);
  if (steps <= 0) return true;
  for (int t0 = t_first; t0 < total_tiles; t0 += 2 * t_stride) {
    const int t1 = t0 + t_stride;
    const int members = t1 < total_tiles ? 2 : 1;
    for (int st = 0; st < steps; ++st) {
      const int chunk = s.carry == CARRY_FWD ? st : s.carry_chunks - 1 - st;
      for (int m = 0; m < members; ++m)
        if (!f(m ? t1 : t0, chunk, m, st, steps)) return false;
    }
  }
  return true;
}

// The epilogue warps of a carry product. For every chunk step: wait for the accumulator, write
// the state it holds to slot (b * NT + state index) of the output (staged through shared memory
// and TMA stores, or stored directly when the layout does not allow that), or after the last
// forward chunk with carry_end the fp32 end state (direct stores); with an aux (the other state
// sequence, same layout) add the warp's share of <state, aux>; unless this was the tile's last step
// multiply the accumulator by lam^C in tensor memory; hand the accumulator back. A tile's
// <state, aux> sum, times aux_dot_scale, goes to tile_partial[part_stride * t + part_off + warp].
template <int BM, int BN, bool PAIR, int SLOTS>
__device__ __forceinline__ void carry_epilogue_warps(const GemmShape& shape, const GemmEpilogue& epi,
                                                     const CUtensorMap* tma_out, const CUtensorMap* tma_aux,
                                                     int m_blocks, int n_blocks, int tiles_per_batch,
                                                     int total_tiles, int t_first, int t_stride, int cta_rows,
                                                     uint32_t tmem_base, uint64_t* tfull, uint64_t* tempty,
                                                     uint32_t leader_tempty, uint8_t* stage, uint64_t* aux_bar,
                                                     volatile int* abort_flag, int site, int part_stride,
                                                     int part_off) {
  constexpr int PART = BN / (EPI_WARPS / 4) < 64 ? 64 : BN / (EPI_WARPS / 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ew = warp - 2;
  const int quad = warp & 3;
  const int part = ew >> 2;
  const bool active = part * PART < BN;
  const bool f32 = epi.out_dtype == ULM_F32;
  const bool staged = epi.staged == EPI_MODE_WARP;
  const bool dot = epi.aux != nullptr;
  const float lamC = fast_exp2((*epi.g) * 1.4426950408889634f * (float)shape.carry_C);
  const int NT = shape.carry_chunks;
  uint8_t* wslots = stage + ew * (SLOTS * 4096);
  uint64_t* wbar = aux_bar + ew * SLOTS;
  const int cw = f32 ? 32 : 64;  // columns of a staged chunk
  int n = 0;                     // staged chunks of this warp so far (slot n % SLOTS)
  int n_issued = 0;              // aux loads issued by this warp (lane 0's count)
  int uses[2] = {0, 0};
  float dg_member[2] = {0.f, 0.f};
  const bool ok = carry_walk(t_first, t_stride, total_tiles, shape,
                             [&](int t, int chunk, int acc, int step, int steps) -> bool {
    const TileCoord tc = decode_tile<BM, BN>(t, shape, m_blocks, n_blocks, tiles_per_batch);
    const uint32_t acc_phase = (uint32_t)(uses[acc]++) & 1u;
    const int row_base = tc.mb * BM + cta_rows + quad * 32;
    const int row = row_base + lane;
    const int col_base = tc.nb * BN + part * PART;
    const bool cols = active && row_base < shape.M && col_base < shape.N;
    const bool last = step == steps - 1;
    const bool to_end = shape.carry == CARRY_FWD && shape.carry_end && chunk == NT - 1;
    const int slot = shape.carry == CARRY_FWD ? chunk + 1 : chunk - 1;
    const int ob = tc.b * NT + slot;  // output (and aux) batch coordinate
    const int nch = (cols && !to_end && staged) ? min(PART / cw, (shape.N - col_base + cw - 1) / cw) : 0;
    if (dot && lane == 0 && nch > 0) {
      bulk_wait_group_read<0>();  // every earlier store of this warp has read its slot
      for (int i = 0; i < nch && i < SLOTS; ++i) {
        epi_aux_issue<SLOTS>(tma_aux, wslots, wbar, n + i, col_base + i * cw, row_base, ob);
        ++n_issued;
      }
    }
    if (!wait_or_abort(&tfull[acc], acc_phase, abort_flag, site)) return false;
    tc_fence_after();
    const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN + part * PART);
    float dg_acc = 0.f;
    if (!cols) {
      // nothing of this tile for this warp: only its barrier arrival below
    } else if (to_end) {
#pragma unroll 1
      for (int c = 0; c < PART; c += 16) {
        float v[16];
        tmem_ld_32x16(taddr + (uint32_t)c, v);
        const int col0 = col_base + c;
        if (row < shape.M) {
          float* o = epi.end_state + (int64_t)tc.b * epi.end_bstride + (int64_t)row * epi.end_ld;
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (col0 + i < shape.N) o[col0 + i] = v[i];
        }
      }
    } else if (staged) {
#pragma unroll 1
      for (int i = 0; i < nch; ++i) {
        const int sl = n % SLOTS;
        const uint32_t parity = (uint32_t)(n / SLOTS) & 1u;
        ++n;
        uint8_t* tile = wslots + sl * 4096;
        if (!dot) {
          if (lane == 0) bulk_wait_group_read<SLOTS - 1>();  // the store of chunk n - SLOTS has read the slot
          __syncwarp();
        } else if (!wait_or_abort(&wbar[sl], parity, abort_flag, site)) {
          return false;
        }
#pragma unroll 1
        for (int h = 0; h < (f32 ? 2 : 4); ++h) {
          float v[16];
          const uint32_t ta = taddr + (uint32_t)(i * cw + 16 * h);
          tmem_ld_32x16(ta, v);
          const int u0 = f32 ? 4 * h : 2 * h;
          if (dot) {
            float p[16];
            if (f32)
              stage_read<true, 16>(tile, lane, u0, p);
            else
              stage_read<false, 16>(tile, lane, u0, p);
            const int c0 = col_base + i * cw + 16 * h;
#pragma unroll
            for (int e = 0; e < 16; ++e)
              if (c0 + e < shape.N) dg_acc = fmaf(p[e], v[e], dg_acc);
          }
          if (f32)
            stage_write<true, 16>(tile, lane, u0, v);
          else
            stage_write<false, 16>(tile, lane, u0, v);
          if (!last) {
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] *= lamC;
            tmem_st_32x16(ta, v);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(tma_out, tile, col_base + i * cw, row_base, ob);
          bulk_commit_group();
          if (dot && i + SLOTS < nch) {
            bulk_wait_group_read<0>();  // the store just issued has read the slot
            epi_aux_issue<SLOTS>(tma_aux, wslots, wbar, n - 1 + SLOTS, col_base + (i + SLOTS) * cw, row_base, ob);
            ++n_issued;
          }
        }
        __syncwarp();
      }
    } else {
#pragma unroll 1
      for (int c = 0; c < PART; c += 16) {
        float v[16];
        tmem_ld_32x16(taddr + (uint32_t)c, v);
        const int col0 = col_base + c;
        if (row < shape.M) {
          const int64_t off = (int64_t)ob * epi.out_bstride + (int64_t)row * epi.ldo + col0;
          const int64_t aoff = (int64_t)ob * epi.aux_bstride + (int64_t)row * epi.ld_aux + col0;
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            if (col0 + e >= shape.N) continue;
            if (f32) {
              reinterpret_cast<float*>(epi.out)[off + e] = v[e];
              if (dot) dg_acc = fmaf(reinterpret_cast<const float*>(epi.aux)[aoff + e], v[e], dg_acc);
            } else {
              reinterpret_cast<__nv_bfloat16*>(epi.out)[off + e] = __float2bfloat16_rn(v[e]);
              if (dot)
                dg_acc = fmaf(__bfloat162float(reinterpret_cast<const __nv_bfloat16*>(epi.aux)[aoff + e]), v[e],
                              dg_acc);
            }
          }
        }
        if (!last) {
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] *= lamC;
          tmem_st_32x16(taddr + (uint32_t)c, v);
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      if (PAIR)
        mbar_arrive_cluster(leader_tempty + (uint32_t)(acc * sizeof(uint64_t)));
      else
        mbar_arrive(&tempty[acc]);
    }
    dg_member[acc] += dg_acc;
    if (last && dot) {
      float d = dg_member[acc];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      if (lane == 0)
        epi.tile_partial[part_stride * (int64_t)t + part_off + ew] =
            d * epi.aux_dot_scale * fast_exp2((*epi.g) * 1.4426950408889634f * epi.aux_dot_pow);
      dg_member[acc] = 0.f;
    }
    return true;
  });
  if (lane == 0) {
    // aux loads still in flight after an abort land before the CTA exits; stores complete
    if (!ok && dot && staged) {
      for (int k = max(0, n_issued - SLOTS); k < n_issued; ++k) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&wbar[k % SLOTS], (uint32_t)(k / SLOTS) & 1u) &&
               globaltimer_ns() - t0 < 100000000ull) {
        }
      }
    }
    bulk_wait_group<0>();
  }
}

// ------------------------------------------------------------------------------------------------
// tensor-core back end

constexpr int TC_BM = 128;
constexpr int TC_BK = 64;
constexpr int TC_THREADS = 64 + 32 * EPI_WARPS;

template <int BN>
struct TcConfig {
  static constexpr int STAGES = BN == 256 ? 3 : 5;
  static constexpr int EPI_SLOTS = 2;
  static constexpr uint32_t A_BYTES = TC_BM * TC_BK * 2;
  static constexpr uint32_t B_BYTES = BN * TC_BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  // stages + staging tiles of the epilogue + 1024 alignment slack + barriers / TMEM slot / flags
  static constexpr uint32_t SMEM_BYTES = STAGES * STAGE_BYTES + epi_smem_bytes(EPI_SLOTS) + 1024 + 512;
};

template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   const __grid_constant__ CUtensorMap tma_a2, const __grid_constant__ CUtensorMap tma_b2,
                   const __grid_constant__ CUtensorMap tma_out, const __grid_constant__ CUtensorMap tma_aux,
                   const GemmShape shape, const GemmEpilogue epi, const int m_blocks, const int n_blocks,
                   const int tiles_per_batch, const int total_tiles) {
  using Cfg = TcConfig<BN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr uint32_t IDESC = idesc_bf16_f32(TC_BM, BN, A_MN, B_MN);
  // descriptor strides: K-major rows are 128 B, 8-row atoms 1024 B apart; MN-major operands keep
  // 64-element M/N blocks of 64 K-rows (8 KB) one after the other
  constexpr uint32_t SBO = 1024;
  constexpr uint32_t MN_LBO = TC_BK * 128;
  // per K=16 step: K-major advances 32 B inside the swizzle row, MN-major advances 16 rows
  constexpr uint32_t A_KSTEP = A_MN ? 16 * 128 : 32;
  constexpr uint32_t B_KSTEP = B_MN ? 16 * 128 : 32;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_stage = smem + STAGES * Cfg::STAGE_BYTES;  // Cfg::EPI_SLOTS staging tiles per epilogue warp
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + epi_smem_bytes(Cfg::EPI_SLOTS));
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* aux_bar = drain + 1;  // up to EPI_MAX_SLOTS per epilogue warp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aux_bar + EPI_MAX_SLOTS * EPI_WARPS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], EPI_WARPS);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < EPI_MAX_SLOTS * EPI_WARPS; ++i) mbar_init(&aux_bar[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
    if (shape.K2 > 0) {
      tma_prefetch_desc(&tma_a2);
      tma_prefetch_desc(&tma_b2);
    }
    if (epi.staged != EPI_MODE_DIRECT) {
      tma_prefetch_desc(&tma_out);
      if (has_tile_aux(epi.kind) || (shape.carry && epi.aux)) tma_prefetch_desc(&tma_aux);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_enter();  // set-up done: wait for the previous kernel's results before touching global memory

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;  // stages issued and possibly not yet consumed (for draining on abort)
      bool ok = true;
      if (shape.carry) {
        ok = carry_walk(blockIdx.x, gridDim.x, total_tiles, shape, [&](int t, int chunk, int, int, int) -> bool {
          const TileCoord tc = decode_tile<TC_BM, BN>(t, shape, m_blocks, n_blocks, tiles_per_batch);
          const int k_lo = chunk * shape.carry_C, k_hi = min(shape.K, k_lo + shape.carry_C);
          for (int kb = k_lo / TC_BK; kb * TC_BK < k_hi; ++kb) {
            if (!wait_or_abort(&empty[stage], phase ^ 1u, abort_flag, DEVERR_GEMM_PRODUCER_WAIT)) return false;
            uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
            uint8_t* sb = sa + Cfg::A_BYTES;
            mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
            const int k0 = kb * TC_BK;
            if (!A_MN) {
              tma_load_3d(&tma_a, sa, &full[stage], k0, tc.mb * TC_BM, tc.b);
            } else {
#pragma unroll
              for (int j = 0; j < TC_BM / 64; ++j)
                tma_load_3d(&tma_a, sa + j * MN_LBO, &full[stage], tc.mb * TC_BM + j * 64, k0, tc.b);
            }
            if (!B_MN) {
              tma_load_3d(&tma_b, sb, &full[stage], k0, tc.nb * BN, tc.b);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j)
                tma_load_3d(&tma_b, sb + j * MN_LBO, &full[stage], tc.nb * BN + j * 64, k0, tc.b);
            }
            issued = min(issued + 1, STAGES);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
          return true;
        });
      }
      const int rounded =
          shape.carry ? 0 : (total_tiles + (int)gridDim.x - 1) / (int)gridDim.x * (int)gridDim.x;
      for (int tt = blockIdx.x; tt < rounded && ok; tt += gridDim.x) {
        const int t = schedule_tile(tt, gridDim.x, total_tiles, shape.balanced);
        if (t < 0) continue;
        const TileCoord tc = decode_tile<TC_BM, BN>(t, shape, m_blocks, n_blocks, tiles_per_batch);
        const int kb0 = tc.k_begin / TC_BK, kb1 = (tc.k_end + TC_BK - 1) / TC_BK;
        const int n1 = kb1 - kb0, nkb = n1 + (shape.K2 + TC_BK - 1) / TC_BK;
        const int ob = shape.ksplit > 1 ? 0 : tc.b;  // operand batch coordinate
        for (int i = 0; i < nkb; ++i) {
          if (!wait_or_abort(&empty[stage], phase ^ 1u, abort_flag, DEVERR_GEMM_PRODUCER_WAIT)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          // k blocks of the first operand pair, then those of the second (shape.K2)
          const bool s2 = i >= n1;
          const CUtensorMap* ma = s2 ? &tma_a2 : &tma_a;
          const CUtensorMap* mbm = s2 ? &tma_b2 : &tma_b;
          const int k0 = (s2 ? i - n1 : kb0 + i) * TC_BK;
          const int oa = s2 ? (shape.a2_batched ? tc.b : 0) : ob;
          const int obb = s2 ? (shape.b2_batched ? tc.b : 0) : ob;
          if (!A_MN) {
            tma_load_3d(ma, sa, &full[stage], k0, tc.mb * TC_BM, oa);
          } else {
#pragma unroll
            for (int j = 0; j < TC_BM / 64; ++j)
              tma_load_3d(ma, sa + j * MN_LBO, &full[stage], tc.mb * TC_BM + j * 64, k0, oa);
          }
          if (!B_MN) {
            tma_load_3d(mbm, sb, &full[stage], k0, tc.nb * BN, obb);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_3d(mbm, sb + j * MN_LBO, &full[stage], tc.nb * BN + j * 64, k0, obb);
          }
          issued = min(issued + 1, STAGES);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // drain: wait (bounded) for the loads still in flight into the last `issued` stages
        for (int i = 0; i < issued; ++i) {
          if (--stage < 0) {
            stage = STAGES - 1;
            phase ^= 1u;
          }
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[stage], phase) && globaltimer_ns() - t0 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      int stage = 0;
      uint32_t phase = 0;
      int j = 0;
      bool ok = true, issued_any = false;
      if (shape.carry) {
        int uses[2] = {0, 0};
        ok = carry_walk(blockIdx.x, gridDim.x, total_tiles, shape, [&](int, int chunk, int acc, int step, int) -> bool {
          const uint32_t acc_phase = (uint32_t)(uses[acc]++) & 1u;
          if (!wait_or_abort(&tempty[acc], acc_phase ^ 1u, abort_flag, DEVERR_GEMM_MMA_WAIT)) return false;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
          const int k_lo = chunk * shape.carry_C, k_hi = min(shape.K, k_lo + shape.carry_C);
          for (int kb = k_lo / TC_BK, i = 0; kb * TC_BK < k_hi; ++kb, ++i) {
            if (!wait_or_abort(&full[stage], phase, abort_flag, DEVERR_GEMM_MMA_WAIT)) return false;
            tc_fence_after();
            const uint32_t sa = smem_u32(smem + stage * Cfg::STAGE_BYTES);
            const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
            for (int kk = 0; kk < TC_BK / 16; ++kk) {
              const uint64_t ad = smem_desc_sw128(sa + kk * A_KSTEP, A_MN ? MN_LBO : 16, SBO);
              const uint64_t bd = smem_desc_sw128(sb + kk * B_KSTEP, B_MN ? MN_LBO : 16, SBO);
              umma_bf16_ss(d_tmem, ad, bd, IDESC, (step > 0 || i > 0 || kk > 0) ? 1u : 0u);
            }
            issued_any = true;
            umma_commit(&empty[stage]);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
          umma_commit(&tfull[acc]);
          return true;
        });
      }
      const int rounded =
          shape.carry ? 0 : (total_tiles + (int)gridDim.x - 1) / (int)gridDim.x * (int)gridDim.x;
      for (int tt = blockIdx.x; tt < rounded && ok; tt += gridDim.x) {
        const int t = schedule_tile(tt, gridDim.x, total_tiles, shape.balanced);
        if (t < 0) continue;
        const TileCoord tc = decode_tile<TC_BM, BN>(t, shape, m_blocks, n_blocks, tiles_per_batch);
        const int kb0 = tc.k_begin / TC_BK, kb1 = (tc.k_end + TC_BK - 1) / TC_BK;
        const int nkb = kb1 - kb0 + (shape.K2 + TC_BK - 1) / TC_BK;
        const int jj = j++;
        const int acc = jj & 1;
        const uint32_t acc_phase = (uint32_t)(jj >> 1) & 1u;
        if (!wait_or_abort(&tempty[acc], acc_phase ^ 1u, abort_flag, DEVERR_GEMM_MMA_WAIT)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int i = 0; i < nkb; ++i) {
          if (!wait_or_abort(&full[stage], phase, abort_flag, DEVERR_GEMM_MMA_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < TC_BK / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(sa + kk * A_KSTEP, A_MN ? MN_LBO : 16, SBO);
            const uint64_t bd = smem_desc_sw128(sb + kk * B_KSTEP, B_MN ? MN_LBO : 16, SBO);
            umma_bf16_ss(d_tmem, ad, bd, IDESC, (i > 0 || kk > 0) ? 1u : 0u);
          }
          issued_any = true;
          umma_commit(&empty[stage]);  // frees the stage once these MMAs have read it
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);  // accumulator ready for the epilogue
      }
      if (!ok && issued_any) {
        umma_commit(drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2.., TMEM lane quadrant = warp % 4) ----------------
    if (shape.carry)
      carry_epilogue_warps<TC_BM, BN, false, Cfg::EPI_SLOTS>(
          shape, epi, &tma_out, &tma_aux, m_blocks, n_blocks, tiles_per_batch, total_tiles, blockIdx.x, gridDim.x,
          0, tmem_base, tfull, tempty, 0u, epi_stage, aux_bar, abort_flag, DEVERR_GEMM_EPILOGUE_WAIT, EPI_WARPS, 0);
    else
      epilogue_warps<TC_BM, BN, false, Cfg::EPI_SLOTS>(shape, epi, &tma_out, &tma_aux, m_blocks, n_blocks, tiles_per_batch, total_tiles,
                                     blockIdx.x, gridDim.x, 0, tmem_base, tfull, tempty, 0u, epi_stage, aux_bar,
                                     abort_flag, DEVERR_GEMM_EPILOGUE_WAIT, EPI_WARPS, 0);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------------
// tensor-core back end, CTA pairs: 256 x 256 tiles with the 2-SM MMA (tcgen05 cta_group::2)
//
// A cluster of two CTAs computes one 256 x 256 tile: each CTA loads its 128 rows of A and its 128
// columns of B (so every SM streams half of B), the leader (cluster rank 0) issues
// tcgen05.mma.cta_group::2 with M = 256, N = 256, and each CTA's TMEM receives its 128 rows. Stage
// hand-off: both CTAs' TMA loads complete on the leader's `full` barrier (the leader posts the
// expected bytes of both), the leader's commit arrives on `empty` / `tfull` of both CTAs, and both
// CTAs' epilogue warps arrive on the leader's `tempty`.

constexpr int TC2_BN = 256;
constexpr int TC2_STAGES = 5;

struct Tc2Config {
  static constexpr uint32_t A_BYTES = 128 * TC_BK * 2;  // this CTA's 128 rows of A
  static constexpr uint32_t B_BYTES = 128 * TC_BK * 2;  // this CTA's 128 columns of B
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t TMEM_COLS = 2 * TC2_BN;
  // two staging tiles per epilogue warp (three would leave room for only four operand stages, which
  // slows the long-K products more than the extra aux load in flight speeds up the fp32 epilogues)
  static constexpr int EPI_SLOTS = 2;
  static constexpr uint32_t SMEM_BYTES = TC2_STAGES * STAGE_BYTES + epi_smem_bytes(EPI_SLOTS) + 1024 + 512;
};

template <bool A_MN, bool B_MN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(TC_THREADS, 1)
    tc2_gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                    const __grid_constant__ CUtensorMap tma_a2, const __grid_constant__ CUtensorMap tma_b2,
                    const __grid_constant__ CUtensorMap tma_out, const __grid_constant__ CUtensorMap tma_aux,
                    const GemmShape shape, const GemmEpilogue epi, const int m_blocks, const int n_blocks,
                    const int tiles_per_batch, const int total_tiles) {
  using Cfg = Tc2Config;
  constexpr int STAGES = TC2_STAGES;
  constexpr int BM = 256, BN = TC2_BN;
  constexpr uint32_t IDESC = idesc_bf16_f32(BM, BN, A_MN, B_MN);
  constexpr uint32_t SBO = 1024;
  constexpr uint32_t MN_LBO = TC_BK * 128;
  constexpr uint32_t A_KSTEP = A_MN ? 16 * 128 : 32;
  constexpr uint32_t B_KSTEP = B_MN ? 16 * 128 : 32;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_stage = smem + STAGES * Cfg::STAGE_BYTES;  // Cfg::EPI_SLOTS staging tiles per epilogue warp
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + epi_smem_bytes(Cfg::EPI_SLOTS));
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* aux_bar = drain + 1;  // up to EPI_MAX_SLOTS per epilogue warp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aux_bar + EPI_MAX_SLOTS * EPI_WARPS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * EPI_WARPS);  // the epilogue warps of both CTAs of the pair
    }
    mbar_init(drain, 1);
    for (int i = 0; i < EPI_MAX_SLOTS * EPI_WARPS; ++i) mbar_init(&aux_bar[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
    if (shape.K2 > 0) {
      tma_prefetch_desc(&tma_a2);
      tma_prefetch_desc(&tma_b2);
    }
    if (epi.staged != EPI_MODE_DIRECT) {
      tma_prefetch_desc(&tma_out);
      if (has_tile_aux(epi.kind) || (shape.carry && epi.aux)) tma_prefetch_desc(&tma_aux);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM of the pair allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_enter();  // set-up done: wait for the previous kernel's results before touching global memory

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer (both CTAs) ----------------
      const uint32_t leader_full = mapa_shared(smem_u32(full), 0);
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      // one stage: k block kb (64 k values) of the first operand pair for tile coordinate tc
      auto load_stage = [&](const TileCoord& tc, int kb) -> bool {
        if (!wait_or_abort(&empty[stage], phase ^ 1u, abort_flag, DEVERR_GEMM2_WAIT)) return false;
        uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
        uint8_t* sb = sa + Cfg::A_BYTES;
        const uint32_t bar = leader_full + (uint32_t)(stage * sizeof(uint64_t));
        if (leader) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
        const int k0 = kb * TC_BK;
        const int row0 = tc.mb * BM + (int)rank * 128;
        const int col0 = tc.nb * BN + (int)rank * 128;
        if (!A_MN) {
          tma_load_3d_pair(&tma_a, sa, bar, k0, row0, tc.b);
        } else {
          tma_load_3d_pair(&tma_a, sa, bar, row0, k0, tc.b);
          tma_load_3d_pair(&tma_a, sa + MN_LBO, bar, row0 + 64, k0, tc.b);
        }
        if (!B_MN) {
          tma_load_3d_pair(&tma_b, sb, bar, k0, col0, tc.b);
        } else {
          tma_load_3d_pair(&tma_b, sb, bar, col0, k0, tc.b);
          tma_load_3d_pair(&tma_b, sb + MN_LBO, bar, col0 + 64, k0, tc.b);
        }
        issued = min(issued + 1, STAGES);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
        return true;
      };
      if (shape.carry) {
        ok = carry_walk(pair, pairs, total_tiles, shape, [&](int t, int chunk, int, int, int) -> bool {
          const TileCoord tc = decode_tile<BM, BN>(t, shape, m_blocks, n_blocks, tiles_per_batch);
          const int k_lo = chunk * shape.carry_C, k_hi = min(shape.K, k_lo + shape.carry_C);
          for (int kb = k_lo / TC_BK; kb * TC_BK < k_hi; ++kb)
            if (!load_stage(tc, kb)) return false;
          return true;
        });
      }
      const int rounded = shape.carry ? 0 : (total_tiles + pairs - 1) / pairs * pairs;
      for (int tt = pair; tt < rounded && ok; tt += pairs) {
        const int t = schedule_tile(tt, pairs, total_tiles, shape.balanced);
        if (t < 0) continue;
        const TileCoord tc = decode_tile<BM, BN>(t, shape, m_blocks, n_blocks, tiles_per_batch);
        const int kb0 = tc.k_begin / TC_BK, kb1 = (tc.k_end + TC_BK - 1) / TC_BK;
        const int n1 = kb1 - kb0, nkb = n1 + (shape.K2 + TC_BK - 1) / TC_BK;
        const int ob = shape.ksplit > 1 ? 0 : tc.b;  // operand batch coordinate
        const int row0 = tc.mb * BM + (int)rank * 128;
        const int col0 = tc.nb * BN + (int)rank * 128;
        for (int i = 0; i < nkb; ++i) {
          if (!wait_or_abort(&empty[stage], phase ^ 1u, abort_flag, DEVERR_GEMM2_WAIT)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          const uint32_t bar = leader_full + (uint32_t)(stage * sizeof(uint64_t));
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
          // k blocks of the first operand pair, then those of the second (shape.K2)
          const bool s2 = i >= n1;
          const CUtensorMap* ma = s2 ? &tma_a2 : &tma_a;
          const CUtensorMap* mbm = s2 ? &tma_b2 : &tma_b;
          const int k0 = (s2 ? i - n1 : kb0 + i) * TC_BK;
          const int oa = s2 ? (shape.a2_batched ? tc.b : 0) : ob;
          const int obb = s2 ? (shape.b2_batched ? tc.b : 0) : ob;
          if (!A_MN) {
            tma_load_3d_pair(ma, sa, bar, k0, row0, oa);
          } else {
            tma_load_3d_pair(ma, sa, bar, row0, k0, oa);
            tma_load_3d_pair(ma, sa + MN_LBO, bar, row0 + 64, k0, oa);
          }
          if (!B_MN) {
            tma_load_3d_pair(mbm, sb, bar, k0, col0, obb);
          } else {
            tma_load_3d_pair(mbm, sb, bar, col0, k0, obb);
            tma_load_3d_pair(mbm, sb + MN_LBO, bar, col0 + 64, k0, obb);
          }
          issued = min(issued + 1, STAGES);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && leader) {
        for (int i = 0; i < issued; ++i) {
          if (--stage < 0) {
            stage = STAGES - 1;
            phase ^= 1u;
          }
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[stage], phase) && globaltimer_ns() - t0 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (leader CTA) ----------------
      int stage = 0;
      uint32_t phase = 0;
      int j = 0;
      bool ok = true, issued_any = false;
      if (shape.carry) {
        int uses[2] = {0, 0};
        ok = carry_walk(pair, pairs, total_tiles, shape, [&](int, int chunk, int acc, int step, int) -> bool {
          const uint32_t acc_phase = (uint32_t)(uses[acc]++) & 1u;
          if (!wait_or_abort(&tempty[acc], acc_phase ^ 1u, abort_flag, DEVERR_GEMM2_WAIT)) return false;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
          const int k_lo = chunk * shape.carry_C, k_hi = min(shape.K, k_lo + shape.carry_C);
          for (int kb = k_lo / TC_BK, i = 0; kb * TC_BK < k_hi; ++kb, ++i) {
            if (!wait_or_abort(&full[stage], phase, abort_flag, DEVERR_GEMM2_WAIT)) return false;
            tc_fence_after();
            const uint32_t sa = smem_u32(smem + stage * Cfg::STAGE_BYTES);
            const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
            for (int kk = 0; kk < TC_BK / 16; ++kk) {
              const uint64_t ad = smem_desc_sw128(sa + kk * A_KSTEP, A_MN ? MN_LBO : 16, SBO);
              const uint64_t bd = smem_desc_sw128(sb + kk * B_KSTEP, B_MN ? MN_LBO : 16, SBO);
              // the first chunk starts the state; later chunks add to the rescaled state
              umma_bf16_ss_pair(d_tmem, ad, bd, IDESC, (step > 0 || i > 0 || kk > 0) ? 1u : 0u);
            }
            issued_any = true;
            umma_commit_pair(&empty[stage], 0x3);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
          umma_commit_pair(&tfull[acc], 0x3);
          return true;
        });
      }
      const int rounded = shape.carry ? 0 : (total_tiles + pairs - 1) / pairs * pairs;
      for (int tt = pair; tt < rounded && ok; tt += pairs) {
        const int t = schedule_tile(tt, pairs, total_tiles, shape.balanced);
        if (t < 0) continue;
        const TileCoord tc = decode_tile<BM, BN>(t, shape, m_blocks, n_blocks, tiles_per_batch);
        const int kb0 = tc.k_begin / TC_BK, kb1 = (tc.k_end + TC_BK - 1) / TC_BK;
        const int nkb = kb1 - kb0 + (shape.K2 + TC_BK - 1) / TC_BK;
        const int jj = j++;
        const int acc = jj & 1;
        const uint32_t acc_phase = (uint32_t)(jj >> 1) & 1u;
        if (!wait_or_abort(&tempty[acc], acc_phase ^ 1u, abort_flag, DEVERR_GEMM2_WAIT)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int i = 0; i < nkb; ++i) {
          if (!wait_or_abort(&full[stage], phase, abort_flag, DEVERR_GEMM2_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < TC_BK / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(sa + kk * A_KSTEP, A_MN ? MN_LBO : 16, SBO);
            const uint64_t bd = smem_desc_sw128(sb + kk * B_KSTEP, B_MN ? MN_LBO : 16, SBO);
            umma_bf16_ss_pair(d_tmem, ad, bd, IDESC, (i > 0 || kk > 0) ? 1u : 0u);
          }
          issued_any = true;
          umma_commit_pair(&empty[stage], 0x3);  // frees this stage in both CTAs
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc], 0x3);  // both halves of the accumulator ready
      }
      if (!ok && issued_any) {
        umma_commit_pair(drain, 0x1);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2.. of both CTAs) ----------------
    if (shape.carry)
      carry_epilogue_warps<BM, BN, true, Cfg::EPI_SLOTS>(
          shape, epi, &tma_out, &tma_aux, m_blocks, n_blocks, tiles_per_batch, total_tiles, pair, pairs,
          (int)rank * 128, tmem_base, tfull, tempty, mapa_shared(smem_u32(tempty), 0), epi_stage, aux_bar,
          abort_flag, DEVERR_GEMM2_WAIT, 2 * EPI_WARPS, (int)rank * EPI_WARPS);
    else
      epilogue_warps<BM, BN, true, Cfg::EPI_SLOTS>(shape, epi, &tma_out, &tma_aux, m_blocks, n_blocks, tiles_per_batch, total_tiles, pair,
                                 pairs, (int)rank * 128, tmem_base, tfull, tempty, mapa_shared(smem_u32(tempty), 0),
                                 epi_stage, aux_bar, abort_flag, DEVERR_GEMM2_WAIT, 2 * EPI_WARPS,
                                 (int)rank * EPI_WARPS);
  }

  tc_fence_before();
  cluster_sync_all();  // all MMAs done and all TMEM reads finished in both CTAs
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------------
// FMA back end

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(256)
    simt_gemm_kernel(const float* __restrict__ A, int64_t lda, int64_t bsA, const float* __restrict__ Bm, int64_t ldb,
                     int64_t bsB, const float* __restrict__ A2, int64_t lda2, int64_t bsA2,
                     const float* __restrict__ B2, int64_t ldb2, int64_t bsB2, const GemmShape shape,
                     const GemmEpilogue epi, const int m_blocks, const int n_blocks, const int tiles_per_batch) {
  constexpr int BM = 64, BN = 64, BK = 16;
  __shared__ float As[BK][BM + 1];
  __shared__ float Bs[BK][BN + 1];
  pdl_enter();
  const TileCoord tc = decode_tile<BM, BN>(blockIdx.x, shape, m_blocks, n_blocks, tiles_per_batch);
  const float* Ab = A + (int64_t)tc.b * bsA;
  const float* Bb = Bm + (int64_t)tc.b * bsB;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) acc[i][jj] = 0.f;

  // the k range of the first operand pair, then all of K2 over the second (when shape.K2 > 0)
  auto segment = [&](const float* Ap, int64_t la, const float* Bp, int64_t lb, int kbeg, int kend) {
  for (int k0 = kbeg; k0 < kend; k0 += BK) {
    for (int i = threadIdx.x; i < BM * BK; i += 256) {
      int mm, kk;
      if (A_MN) { kk = i / BM; mm = i % BM; } else { mm = i / BK; kk = i % BK; }
      const int gm = tc.mb * BM + mm, gk = k0 + kk;
      float val = 0.f;
      if (gm < shape.M && gk < kend) val = A_MN ? Ap[(int64_t)gk * la + gm] : Ap[(int64_t)gm * la + gk];
      As[kk][mm] = val;
    }
    for (int i = threadIdx.x; i < BN * BK; i += 256) {
      int nn, kk;
      if (B_MN) { kk = i / BN; nn = i % BN; } else { nn = i / BK; kk = i % BK; }
      const int gn = tc.nb * BN + nn, gk = k0 + kk;
      float val = 0.f;
      if (gn < shape.N && gk < kend) val = B_MN ? Bp[(int64_t)gk * lb + gn] : Bp[(int64_t)gn * lb + gk];
      Bs[kk][nn] = val;
    }
    __syncthreads();
    // two-level sum: each 16-deep slice in its own partial, then into the accumulator (the rounding
    // error of a k-long dot product grows with k / 16 + 16 instead of k)
    float part[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) part[i][jj] = 0.f;
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) bv[jj] = Bs[kk][tx + 16 * jj];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          if (shape.k_in_order)
            acc[i][jj] = fmaf(a[i], bv[jj], acc[i][jj]);
          else
            part[i][jj] = fmaf(a[i], bv[jj], part[i][jj]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) acc[i][jj] += part[i][jj];
    __syncthreads();
  }
  };
  if (shape.carry) {
    // carry product: the 64 x 64 state tile stays in registers across the chunks; after each chunk
    // it is written to its slot (or the end state), dotted with the aux states, and rescaled
    const int NT = shape.carry_chunks, steps = carry_steps(shape);
    const float lamC = expf(*epi.g * (float)shape.carry_C);
    const bool dot = epi.aux != nullptr;
    float dgp = 0.f;
    for (int step = 0; step < steps; ++step) {
      const int chunk = shape.carry == CARRY_FWD ? step : NT - 1 - step;
      segment(Ab, lda, Bb, ldb, chunk * shape.carry_C, min(shape.K, (chunk + 1) * shape.carry_C));
      const bool to_end = shape.carry == CARRY_FWD && shape.carry_end && chunk == NT - 1;
      const int64_t ob = (int64_t)tc.b * NT + (shape.carry == CARRY_FWD ? chunk + 1 : chunk - 1);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = tc.mb * BM + ty + 16 * i;
        if (row >= shape.M) continue;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int col = tc.nb * BN + tx + 16 * jj;
          if (col >= shape.N) continue;
          const float v = acc[i][jj];
          if (to_end) {
            epi.end_state[(int64_t)tc.b * epi.end_bstride + (int64_t)row * epi.end_ld + col] = v;
            continue;
          }
          const int64_t off = ob * epi.out_bstride + (int64_t)row * epi.ldo + col;
          const int64_t aoff = ob * epi.aux_bstride + (int64_t)row * epi.ld_aux + col;
          if (epi.out_dtype == ULM_F32) {
            reinterpret_cast<float*>(epi.out)[off] = v;
            if (dot) dgp = fmaf(reinterpret_cast<const float*>(epi.aux)[aoff], v, dgp);
          } else {
            reinterpret_cast<__nv_bfloat16*>(epi.out)[off] = __float2bfloat16_rn(v);
            if (dot) dgp = fmaf(__bfloat162float(reinterpret_cast<const __nv_bfloat16*>(epi.aux)[aoff]), v, dgp);
          }
        }
      }
      if (step + 1 < steps) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) acc[i][jj] *= lamC;
      }
    }
    if (dot) {
      // fixed-order block reduction, one partial per tile (slots 1..3 of the tile are zero)
      __shared__ float cred[256];
      cred[threadIdx.x] = dgp;
      __syncthreads();
      for (int stride = 128; stride > 0; stride >>= 1) {
        if ((int)threadIdx.x < stride) cred[threadIdx.x] += cred[threadIdx.x + stride];
        __syncthreads();
      }
      if (threadIdx.x < 4)
        epi.tile_partial[4 * (int64_t)blockIdx.x + threadIdx.x] =
            threadIdx.x == 0 ? cred[0] * epi.aux_dot_scale * expf(*epi.g * epi.aux_dot_pow) : 0.f;
    }
    return;
  }
  segment(Ab, lda, Bb, ldb, tc.k_begin, tc.k_end);
  if (shape.K2 > 0)
    segment(A2 + (shape.a2_batched ? (int64_t)tc.b * bsA2 : 0), lda2, B2 + (shape.b2_batched ? (int64_t)tc.b * bsB2 : 0),
            ldb2, 0, shape.K2);
  if (epi.kind == EPI_LSE) {
    // per row: (max, sum exp) over this tile's columns, merged across the 16 lanes of the row
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = tc.mb * BM + ty + 16 * i;
      const bool rv = row < shape.M && row < epi.rows_valid;
      const int64_t tgt = rv ? epi.targets[row] : -1;
      float m = -INFINITY, sm = 0.f;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int col = tc.nb * BN + tx + 16 * jj;
        if (rv && col < shape.N) {
          const float v = acc[i][jj];
          const float nm = fmaxf(m, v);
          sm = sm * expf(m - nm) + expf(v - nm);
          m = nm;
          if ((int64_t)col == tgt) epi.tile_partial[row] = v;
        }
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        const float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, sm, o);
        const float nm = fmaxf(m, om);
        sm = (nm == -INFINITY) ? 0.f : sm * expf(m - nm) + os * expf(om - nm);
        m = nm;
      }
      if (tx == 0 && rv) {
        float* pp = epi.row_partial + ((int64_t)row * epi.part_ld + tc.nb) * 2;
        pp[0] = m;
        pp[1] = sm;
      }
    }
    return;
  }
  const bool decay = epi.kind == EPI_DECAY || epi.kind == EPI_DECAY_DG;
  const float g = decay ? *epi.g : 0.f;
  float dg_acc = 0.f;
  float rowsum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = tc.mb * BM + ty + 16 * i;
    if (row >= shape.M) continue;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int col = tc.nb * BN + tx + 16 * jj;
      if (col >= shape.N) continue;
      float v = acc[i][jj];
      if (epi.kind == EPI_DECAY_DG && col < row) {
        const float p = reinterpret_cast<const float*>(epi.aux)[(int64_t)tc.b * epi.aux_bstride +
                                                                (int64_t)row * epi.ld_aux + col];
        dg_acc = fmaf((float)(row - col) * p, v, dg_acc);
      }
      if (decay) v = (col <= row) ? v * expf(g * (float)(row - col)) : 0.f;
      if (epi.kind == EPI_ROW_DECAY) v *= expf(*epi.g * (epi.rd_a + epi.rd_s * (float)row));
      if (epi.kind == EPI_STORE_ADD) {
        const int64_t ai = (int64_t)tc.b * epi.aux_bstride + (int64_t)row * epi.ld_aux + col;
        v += epi.out_dtype == ULM_F32 ? reinterpret_cast<const float*>(epi.aux)[ai]
                                      : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(epi.aux)[ai]);
      }
      if (epi.kind == EPI_RELU2) {
        const float a = v + reinterpret_cast<const float*>(epi.aux)[col];
        v = a > 0.f ? a * a : 0.f;
        rowsum[i] += v;
      }
      if (epi.kind == EPI_CE_GRAD) {
        const int64_t tgt = row < epi.rows_valid ? epi.targets[row] : -1;
        v = tgt >= 0 ? (expf(v - epi.row_lse[row]) - ((int64_t)col == tgt ? 1.f : 0.f)) * (*epi.scale) : 0.f;
      }
      const int64_t off = (int64_t)tc.b * epi.out_bstride + (int64_t)row * epi.ldo + col;
      if (epi.out_dtype == ULM_F32)
        reinterpret_cast<float*>(epi.out)[off] = v;
      else
        reinterpret_cast<__nv_bfloat16*>(epi.out)[off] = __float2bfloat16_rn(v);
    }
  }
  if (epi.kind == EPI_RELU2 && epi.row_partial) {
    // the 16 threads sharing a row (same ty, tx = 0..15) are 16 consecutive lanes of one warp
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float rs = rowsum[i];
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, o);
      const int row = tc.mb * BM + ty + 16 * i;
      if (tx == 0 && row < shape.M) epi.row_partial[((int64_t)tc.b * shape.M + row) * epi.part_ld + tc.nb] = rs;
    }
  }
  if (epi.kind == EPI_DECAY_DG) {
    // fixed-order block reduction, one partial per tile (slots 1..3 of the tile are zero)
    __shared__ float red[256];
    red[threadIdx.x] = dg_acc;
    __syncthreads();
    for (int stride = 128; stride > 0; stride >>= 1) {
      if ((int)threadIdx.x < stride) red[threadIdx.x] += red[threadIdx.x + stride];
      __syncthreads();
    }
    if (threadIdx.x < 4) epi.tile_partial[4 * (int64_t)blockIdx.x + threadIdx.x] = threadIdx.x == 0 ? red[0] : 0.f;
  }
}

// ------------------------------------------------------------------------------------------------
// host side

// whether large products use the CTA-pair (2-SM MMA) kernel; ulm_set_gemm_pairs switches it
static int g_gemm_pairs = 1;

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

namespace {

// 3-D tiled map over (inner, rows, batch) of a bf16 operand with a 128-byte swizzle.
int make_tmap(CUtensorMap* map, const Operand& op, int batches, uint32_t box_inner, uint32_t box_rows) {
  auto fn = encode_tiled();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return ULM_ERR_UNSUPPORTED;
  }
  cuuint64_t dims[3] = {(cuuint64_t)op.inner, (cuuint64_t)op.rows, (cuuint64_t)batches};
  cuuint64_t strides[2] = {(cuuint64_t)op.ld * 2, (cuuint64_t)op.bstride * 2};
  cuuint32_t box[3] = {box_inner, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(op.ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): inner=%lld rows=%lld ld=%lld", (int)r, (long long)op.inner,
              (long long)op.rows, (long long)op.ld);
    return ULM_ERR_CUDA;
  }
  return ULM_OK;
}

// 3-D map over (cols, rows, batch) of an epilogue array (output or tile aux) whose boxes are the
// staging tiles of EPI_MODE_WARP: 32 rows x 128 bytes, 128-byte swizzle.
bool make_epi_tmap(CUtensorMap* map, int mode, const void* ptr, int dtype, int64_t cols, int64_t rows, int batches,
                   int64_t ld, int64_t bstride) {
  auto fn = encode_tiled();
  if (!fn || !ptr) return false;
  const bool f32 = dtype == ULM_F32;
  const int64_t es = f32 ? 4 : 2;
  if (!is_aligned16(ptr) || (ld * es) % 16 != 0) return false;
  const int64_t bs_bytes = batches > 1 ? bstride * es : rows * ld * es;
  if (bs_bytes % 16 != 0 || bs_bytes <= 0) return false;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batches};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * es), (cuuint64_t)bs_bytes};
  (void)mode;
  cuuint32_t box[3] = {f32 ? 32u : 64u, 32u, 1};  // 32 rows x 128 bytes
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = fn(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                  const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Tile order of a persistent launch over `total` tiles on P CTAs (pairs): the balanced snake order
// for causal k-range products with at most 4 tiles per CTA (the idle tail of uneven k ranges
// dominates there); index order otherwise (keeps concurrent tiles within few batch rows, L2).
GemmShape with_schedule(const GemmShape& s, int total, int P) {
  GemmShape r = s;
  r.balanced = (s.causal == CAUSAL_KLOWER || s.causal == CAUSAL_KUPPER) && total <= 4 * P ? 1 : 0;
  return r;
}

// library-wide epilogue layout of the tensor-core kernels (ulm_set_epilogue_mode)
static int g_epi_mode = EPI_MODE_WARP;

// Tensor maps of the staged epilogue; falls back to direct stores when the layout does not allow it.
void prepare_epilogue(GemmEpilogue& e, const GemmShape& s, CUtensorMap* tout, CUtensorMap* taux) {
  memset(tout, 0, sizeof(CUtensorMap));
  memset(taux, 0, sizeof(CUtensorMap));
  const int mode = g_epi_mode;
  // a carry product writes one state per chunk slot: its output (and aux) hold batches * chunks
  const int ob = s.carry ? s.batches * s.carry_chunks : s.batches;
  bool ok = mode != EPI_MODE_DIRECT && e.vec_ok && s.N >= 32 &&
            make_epi_tmap(tout, mode, e.out, e.out_dtype, s.N, s.M, ob, e.ldo, e.out_bstride);
  if (ok && (has_tile_aux(e.kind) || (s.carry && e.aux)))
    ok = make_epi_tmap(taux, mode, e.aux, e.out_dtype, s.N, s.M, ob, e.ld_aux, e.aux_bstride);
  e.staged = ok ? mode : EPI_MODE_DIRECT;
}

// Tensor maps of the second operand pair (zeroed and unused without one); a pair member with
// batch stride 0 is one matrix shared by all batch rows.
int make_second_pair(CUtensorMap* ta2, CUtensorMap* tb2, const Operand* A2, const Operand* B2, int batches,
                     uint32_t a_rows, uint32_t b_rows, bool a_mn, bool b_mn) {
  memset(ta2, 0, sizeof(CUtensorMap));
  memset(tb2, 0, sizeof(CUtensorMap));
  if (!A2) return ULM_OK;
  if (int rc = make_tmap(ta2, *A2, A2->bstride ? batches : 1, 64, a_mn ? 64 : a_rows)) return rc;
  return make_tmap(tb2, *B2, B2->bstride ? batches : 1, 64, b_mn ? 64 : b_rows);
}

template <int BN, bool A_MN, bool B_MN>
int launch_tc(const Operand& A, const Operand& B, const Operand* A2, const Operand* B2, const GemmShape& s,
              const GemmEpilogue& e_in, cudaStream_t st) {
  using Cfg = TcConfig<BN>;
  CUtensorMap ta, tb, ta2, tb2, tout, taux;
  const int ob = s.ksplit > 1 ? 1 : s.batches;  // split-K operands are not batched
  int rc = make_tmap(&ta, A, ob, 64, A_MN ? 64 : TC_BM);
  if (rc) return rc;
  rc = make_tmap(&tb, B, ob, 64, B_MN ? 64 : BN);
  if (rc) return rc;
  if ((rc = make_second_pair(&ta2, &tb2, A2, B2, s.batches, TC_BM, BN, A_MN, B_MN))) return rc;
  GemmEpilogue e = e_in;
  prepare_epilogue(e, s, &tout, &taux);
  const int dev = current_device();
  static bool configured[64] = {};
  if (dev < 0 || dev >= 64) {
    set_error("device ordinal %d out of range", dev);
    return ULM_ERR_INVALID;
  }
  if (!configured[dev]) {
    ULM_CUDA_TRY(cudaFuncSetAttribute(tc_gemm_kernel<BN, A_MN, B_MN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)Cfg::SMEM_BYTES));
    configured[dev] = true;
  }
  const int m_blocks = (int)cdiv(s.M, TC_BM), n_blocks = (int)cdiv(s.N, BN);
  const int tpb = tiles_per_batch_host(s, TC_BM, BN, m_blocks, n_blocks);
  const int64_t total64 = (int64_t)tpb * s.batches;
  ULM_REQUIRE(total64 < (1ll << 31), "too many tiles (%lld)", (long long)total64);
  const int total = (int)total64;
  if (total == 0) return ULM_OK;
  const int grid = total < sm_count(dev) ? total : sm_count(dev);
  const GemmShape sb = with_schedule(s, total, grid);
  return launch_pdl(tc_gemm_kernel<BN, A_MN, B_MN>, dim3(grid), dim3(TC_THREADS), Cfg::SMEM_BYTES, st, ta, tb, ta2,
                    tb2, tout, taux, sb, e, m_blocks, n_blocks, tpb, total);
}

template <int BN>
int dispatch_tc_major(const Operand& A, const Operand& B, const Operand* A2, const Operand* B2, const GemmShape& s,
                      const GemmEpilogue& e, cudaStream_t st) {
  if (!A.mn_major && !B.mn_major) return launch_tc<BN, false, false>(A, B, A2, B2, s, e, st);
  if (!A.mn_major && B.mn_major) return launch_tc<BN, false, true>(A, B, A2, B2, s, e, st);
  if (A.mn_major && !B.mn_major) return launch_tc<BN, true, false>(A, B, A2, B2, s, e, st);
  return launch_tc<BN, true, true>(A, B, A2, B2, s, e, st);
}

template <bool A_MN, bool B_MN>
int launch_tc2(const Operand& A, const Operand& B, const Operand* A2, const Operand* B2, const GemmShape& s,
               const GemmEpilogue& e_in, cudaStream_t st) {
  using Cfg = Tc2Config;
  CUtensorMap ta, tb, ta2, tb2, tout, taux;
  const int ob = s.ksplit > 1 ? 1 : s.batches;  // split-K operands are not batched
  int rc = make_tmap(&ta, A, ob, 64, A_MN ? 64 : 128);
  if (rc) return rc;
  rc = make_tmap(&tb, B, ob, 64, B_MN ? 64 : 128);
  if (rc) return rc;
  if ((rc = make_second_pair(&ta2, &tb2, A2, B2, s.batches, 128, 128, A_MN, B_MN))) return rc;
  GemmEpilogue e = e_in;
  prepare_epilogue(e, s, &tout, &taux);
  const int dev = current_device();
  static bool configured[64] = {};
  if (dev < 0 || dev >= 64) {
    set_error("device ordinal %d out of range", dev);
    return ULM_ERR_INVALID;
  }
  if (!configured[dev]) {
    ULM_CUDA_TRY(cudaFuncSetAttribute(tc2_gemm_kernel<A_MN, B_MN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)Cfg::SMEM_BYTES));
    configured[dev] = true;
  }
  const int m_blocks = (int)cdiv(s.M, 256), n_blocks = (int)cdiv(s.N, TC2_BN);
  const int tpb = tiles_per_batch_host(s, 256, TC2_BN, m_blocks, n_blocks);
  const int64_t total64 = (int64_t)tpb * s.batches;
  ULM_REQUIRE(total64 < (1ll << 31), "too many tiles (%lld)", (long long)total64);
  const int total = (int)total64;
  if (total == 0) return ULM_OK;
  const int max_pairs = sm_count(dev) / 2;
  const int pairs = total < max_pairs ? total : max_pairs;
  const GemmShape sb = with_schedule(s, total, pairs);
  return launch_pdl(tc2_gemm_kernel<A_MN, B_MN>, dim3(2 * pairs), dim3(TC_THREADS), Cfg::SMEM_BYTES, st, ta, tb, ta2,
                    tb2, tout, taux, sb, e, m_blocks, n_blocks, tpb, total);
}

int dispatch_tc2(const Operand& A, const Operand& B, const Operand* A2, const Operand* B2, const GemmShape& s,
                 const GemmEpilogue& e, cudaStream_t st) {
  if (!A.mn_major && !B.mn_major) return launch_tc2<false, false>(A, B, A2, B2, s, e, st);
  if (!A.mn_major && B.mn_major) return launch_tc2<false, true>(A, B, A2, B2, s, e, st);
  if (A.mn_major && !B.mn_major) return launch_tc2<true, false>(A, B, A2, B2, s, e, st);
  return launch_tc2<true, true>(A, B, A2, B2, s, e, st);
}

template <bool A_MN, bool B_MN>
int launch_simt(const Operand& A, const Operand& B, const Operand* A2, const Operand* B2, const GemmShape& s,
                const GemmEpilogue& e, cudaStream_t st) {
  const int m_blocks = (int)cdiv(s.M, 64), n_blocks = (int)cdiv(s.N, 64);
  const int tpb = tiles_per_batch_host(s, 64, 64, m_blocks, n_blocks);
  const int64_t total = (int64_t)tpb * s.batches;
  ULM_REQUIRE(total < (1ll << 31), "too many tiles (%lld)", (long long)total);
  if (total == 0) return ULM_OK;
  const bool split = s.ksplit > 1;  // split-K operands are not batched
  simt_gemm_kernel<A_MN, B_MN><<<(unsigned)total, 256, 0, st>>>(
      static_cast<const float*>(A.ptr), A.ld, split ? 0 : A.bstride, static_cast<const float*>(B.ptr), B.ld,
      split ? 0 : B.bstride, A2 ? static_cast<const float*>(A2->ptr) : nullptr, A2 ? A2->ld : 0,
      A2 ? A2->bstride : 0, B2 ? static_cast<const float*>(B2->ptr) : nullptr, B2 ? B2->ld : 0,
      B2 ? B2->bstride : 0, s, e, m_blocks, n_blocks, tpb);
  ULM_LAUNCH_CHECK("simt_gemm_kernel");
  return ULM_OK;
}

}  // namespace

int run_gemm2(const Operand& A, const Operand& B, const Operand* A2, const Operand* B2, const GemmShape& s_in,
              const GemmEpilogue& e, cudaStream_t stream) {
  GemmShape s = s_in;
  if (!A2 || !B2 || s.K2 <= 0) {
    A2 = B2 = nullptr;
    s.K2 = 0;
  } else {
    ULM_REQUIRE(A2->ptr && B2->ptr, "null second operand");
    ULM_REQUIRE(A2->dtype == A.dtype && B2->dtype == B.dtype, "the second operand pair must have the first's type");
    ULM_REQUIRE(A2->mn_major == A.mn_major && B2->mn_major == B.mn_major,
                "the second operand pair must have the first's storage orders");
    ULM_REQUIRE(s.ksplit <= 1, "split K with a second operand pair is not supported");
    s.a2_batched = A2->bstride != 0;
    s.b2_batched = B2->bstride != 0;
    if (A2->dtype == ULM_BF16) {
      ULM_REQUIRE(is_aligned16(A2->ptr) && is_aligned16(B2->ptr), "bf16 operands must be 16-byte aligned");
      ULM_REQUIRE(A2->ld % 8 == 0 && B2->ld % 8 == 0 && A2->bstride % 8 == 0 && B2->bstride % 8 == 0,
                  "bf16 operand strides must be multiples of 8 elements");
      ULM_REQUIRE(A2->ld >= A2->inner && B2->ld >= B2->inner, "row stride shorter than the row");
    }
  }
  ULM_REQUIRE(A.ptr && B.ptr && (e.out || e.kind == EPI_LSE), "null operand or output pointer");
  ULM_REQUIRE((e.kind != EPI_LSE && e.kind != EPI_CE_GRAD) ||
                  (e.targets && s.batches == 1 && (e.kind == EPI_CE_GRAD ? e.row_lse && e.scale
                                                                         : e.row_partial && e.tile_partial)),
              "cross-entropy epilogue needs targets, one batch row and its row buffers");
  ULM_REQUIRE(s.batches >= 0 && s.M >= 0 && s.N >= 0 && s.K >= 0, "negative extent");
  ULM_REQUIRE(A.dtype == B.dtype, "A and B must have the same element type");
  ULM_REQUIRE(e.out_dtype == ULM_F32 || e.out_dtype == ULM_BF16, "bad output dtype");
  ULM_REQUIRE(e.kind == EPI_STORE || e.kind == EPI_STORE_ADD || e.kind == EPI_RELU2 || e.kind == EPI_LSE ||
                  e.kind == EPI_CE_GRAD || e.g,
              "decay epilogue needs g");
  ULM_REQUIRE(e.kind != EPI_RELU2 || e.aux, "EPI_RELU2 needs the bias");
  ULM_REQUIRE(e.kind != EPI_DECAY_DG || (e.aux && e.tile_partial), "EPI_DECAY_DG needs aux and tile_partial");
  ULM_REQUIRE(e.kind != EPI_STORE_ADD || e.aux, "EPI_STORE_ADD needs the addend (in the output's type)");
  if (s.causal == CAUSAL_KLOWER || s.causal == CAUSAL_KUPPER)
    ULM_REQUIRE(s.M == s.K, "causal k range needs a square (M == K) problem");
  if (s.carry) {
    ULM_REQUIRE(s.carry == CARRY_FWD || s.carry == CARRY_REV, "bad carry mode");
    ULM_REQUIRE(s.causal == CAUSAL_NONE && s.ksplit <= 1 && s.K2 == 0 && e.kind == EPI_STORE && e.g,
                "a carry product is a plain product (no causal range, split K or second pair) with EPI_STORE and g");
    ULM_REQUIRE(s.carry_C > 0 && s.carry_chunks >= 1 && (int64_t)s.carry_C * (s.carry_chunks - 1) < s.K &&
                    (int64_t)s.carry_C * s.carry_chunks >= s.K,
                "carry chunks must cover K");
    ULM_REQUIRE(s.carry_chunks == 1 || s.carry_C % 64 == 0, "carry chunk length must be a multiple of 64");
    ULM_REQUIRE(!s.carry_end || (s.carry == CARRY_FWD && e.end_state), "carry_end needs CARRY_FWD and end_state");
    ULM_REQUIRE(!e.aux || e.tile_partial, "a carry aux dot needs tile_partial");
  }
  ULM_REQUIRE(s.ksplit <= 1 || (s.causal == CAUSAL_NONE && s.ksplit == s.batches &&
                                 (int64_t)(s.ksplit - 1) * ksplit_chunk(s.K, s.ksplit) < s.K),
              "split K needs a non-causal product, batches == ksplit and no empty k range");
  if (s.batches == 0 || s.M == 0 || s.N == 0) return ULM_OK;
  ULM_REQUIRE(s.K > 0, "empty contraction");
  if (A.dtype == ULM_BF16) {
    ULM_REQUIRE(is_aligned16(A.ptr) && is_aligned16(B.ptr), "bf16 operands must be 16-byte aligned");
    ULM_REQUIRE(A.ld % 8 == 0 && B.ld % 8 == 0 && A.bstride % 8 == 0 && B.bstride % 8 == 0,
                "bf16 operand strides must be multiples of 8 elements (lda=%lld ldb=%lld)", (long long)A.ld,
                (long long)B.ld);
    ULM_REQUIRE(A.ld >= A.inner && B.ld >= B.inner, "row stride shorter than the row");
    if (s.N >= 256 && s.M >= 256 && g_gemm_pairs) return dispatch_tc2(A, B, A2, B2, s, e, stream);
    if (s.N >= 256) return dispatch_tc_major<256>(A, B, A2, B2, s, e, stream);
    return dispatch_tc_major<128>(A, B, A2, B2, s, e, stream);
  }
  ULM_REQUIRE(A.dtype == ULM_F32, "operands must be bf16 or fp32");
  if (!A.mn_major && !B.mn_major) return launch_simt<false, false>(A, B, A2, B2, s, e, stream);
  if (!A.mn_major && B.mn_major) return launch_simt<false, true>(A, B, A2, B2, s, e, stream);
  if (A.mn_major && !B.mn_major) return launch_simt<true, false>(A, B, A2, B2, s, e, stream);
  return launch_simt<true, true>(A, B, A2, B2, s, e, stream);
}

int run_gemm(const Operand& A, const Operand& B, const GemmShape& s, const GemmEpilogue& e, cudaStream_t stream) {
  return run_gemm2(A, B, nullptr, nullptr, s, e, stream);
}

}  // namespace ulm
