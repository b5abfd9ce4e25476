// Batched GEMM engine shared by every contraction of the fast-memory path.
//
//   C[b][m][n] = sum_k A[b][m][k] * B[b][n][k]          (per batch row b)
//
// A and B may each be stored K-major ([m][k], k contiguous) or MN-major ([k][m], m contiguous), so
// the transposed products of the backward need no transposition pass. A causal mode restricts the
// work to the triangle the fast memory needs:
//   CAUSAL_NLOWER : only tiles with columns n <= rows m (decayed scores, s <= t)
//   CAUSAL_KLOWER : the k range of a row block stops at the block's last row (forward read)
//   CAUSAL_KUPPER : the k range of a row block starts at the block's first row (reversed read)
// and a fused epilogue writes the tile (EPI_STORE), the decayed causal score lam^(m-n) * acc
// masked to n <= m (EPI_DECAY), or that score plus the per-tile partial of
// sum (m-n) * aux[m][n] * acc[m][n] (EPI_DECAY_DG, the score gradient's share of d/dg).
//
// Two back ends share the tile decomposition: a tcgen05/TMA/TMEM tensor-core kernel for bf16
// operands (fp32 accumulation) and an fp32 FMA kernel for the 1e-5 parity mode.
#pragma once

#include "common.cuh"

namespace ulm {

enum { CAUSAL_NONE = 0, CAUSAL_KLOWER = 1, CAUSAL_KUPPER = 2, CAUSAL_NLOWER = 3 };
enum { EPI_STORE = 0, EPI_DECAY = 1, EPI_DECAY_DG = 2, EPI_STORE_ADD = 3, EPI_RELU2 = 4, EPI_LSE = 5, EPI_CE_GRAD = 6,
       EPI_ROW_DECAY = 7 };

// Carry products (GemmShape.carry): the k dimension is time, cut into chunks of carry_C positions,
// and the accumulator of an (M x N) tile is a state that runs across the chunks,
//   forward : S_{c+1} = lam^C S_c + A_c B_c^T   for chunks c = 0, 1, ..., written as S_1, S_2, ...
//   reverse : R_{c-1} = lam^C R_c + A_c B_c^T   for chunks c = NT-1, ..., 1, written as R_{NT-2}, ...
// (A_c, B_c: the chunk's k range of the operands). After each chunk the epilogue writes the state
// to slot (b * NT + state index) of the output, multiplies the accumulator by lam^C in tensor
// memory and hands it back, so the state never leaves the SM between chunks.
enum { CARRY_NONE = 0, CARRY_FWD = 1, CARRY_REV = 2 };

struct GemmShape {
  int batches, M, N, K;
  int causal;
  // set by the tensor-core launch: 1 = causal k-range tiles in decreasing-work order, taken in
  // snake order (schedule_tile); 0 = index order (batch rows consecutive)
  int balanced;
  // > 1: split-K product. The operands are single (not batched); "batch" b = 0 .. ksplit - 1 of the
  // output takes the k range [b * kc, min(K, (b + 1) * kc)), kc = K / ksplit rounded up to 64.
  // ksplit must equal batches. The caller sums the partial outputs.
  int ksplit;
  // second operand pair (run_gemm2): K2 more k steps after the first pair's range, over A2 / B2;
  // a2_batched / b2_batched (set by run_gemm2) say whether they have a batch stride
  int K2;
  int a2_batched, b2_batched;
  // carry products: CARRY_FWD / CARRY_REV, chunk length (a multiple of 64 unless there is one chunk)
  // and chunk count (K = carry_C * carry_chunks); CARRY_FWD with carry_end also runs the last
  // chunk, whose state goes to GemmEpilogue.end_state instead of a slot
  int carry = 0;
  int carry_C = 0;
  int carry_chunks = 0;
  int carry_end = 0;
  // fp32 FMA back end: 1 = one running sum over k in order (run.c's matmul order, for the decode
  // steps' token identity); 0 = each 16-deep k slice summed apart, then added (smaller rounding)
  int k_in_order = 0;
};

// Chunk steps a carry tile runs.
__host__ __device__ inline int carry_steps(const GemmShape& s) {
  if (s.carry == CARRY_FWD) return s.carry_end ? s.carry_chunks : s.carry_chunks - 1;
  return s.carry_chunks - 1;
}

__host__ __device__ inline int ksplit_chunk(int K, int ksplit) { return ((K + ksplit - 1) / ksplit + 63) / 64 * 64; }

struct GemmEpilogue {
  int kind;            // EPI_STORE / EPI_DECAY
  int out_dtype;       // ULM_F32 / ULM_BF16
  void* out;
  int64_t ldo;         // row stride of the output, elements
  int64_t out_bstride; // batch stride of the output, elements
  const float* g;      // log decay (device scalar), EPI_DECAY / EPI_DECAY_DG
  int vec_ok;          // output and aux rows are 16-byte aligned for every tile (set by the host)
  // EPI_STORE_ADD: out = acc + aux (aux in the output's type and layout).
  // EPI_RELU2: out = relu(acc + bias[n])^2, bias = aux (fp32, one value per output column).
  // EPI_DECAY_DG: aux = the forward's decayed scores P (same layout and type as the output); each
  // epilogue warp adds sum (m-n) * P[m][n] * acc[m][n] over its part of a tile and writes it to its
  // own slot of tile_partial (d/dg of the fast read, no atomics; decay_dg_partials slots in all)
  const void* aux;
  int64_t ld_aux, aux_bstride;
  float* tile_partial;
  // EPI_RELU2 only, optional: row_partial[row * part_ld + j] = sum of the row's outputs in column
  // block j (blocks of 128 or 64 columns depending on the back end; part_ld >= N / 64; unused
  // slots untouched)
  float* row_partial;
  int part_ld;
  // set by the tensor-core launch: stage output chunks in shared memory and write them (and read a
  // tile aux) with TMA tensor copies
  int staged;
  // cross-entropy epilogues over logits = acc (one batch row; row r has class targets[r], -1 =
  // ignored):
  // EPI_LSE: nothing is stored; row_partial[(r * part_ld + j) * 2 + {0, 1}] = (max, sum exp(x - max))
  //   of the row's logits in column block j (as for EPI_RELU2), tile_partial[r] = the logit of
  //   column targets[r];
  // EPI_CE_GRAD: out = (exp(acc - row_lse[r]) - [col == targets[r]]) * (*scale), 0 for ignored rows.
  const int64_t* targets = nullptr;
  const float* row_lse = nullptr;
  const float* scale = nullptr;
  int rows_valid = 0;  // rows of the product (bound for targets / row_lse reads)
  // EPI_ROW_DECAY: out = lam^(rd_a + rd_s * row) * acc (row = the row inside its batch row)
  float rd_a = 0.f, rd_s = 0.f;
  // carry products: optional tile aux (the other state sequence, same layout and type as the
  // output) whose elementwise product with each written state is summed per warp into
  // tile_partial (scaled by aux_dot_scale * lam^aux_dot_pow); optional fp32 end state (batch
  // stride end_bstride, row stride end_ld) for CARRY_FWD with carry_end
  float aux_dot_scale = 0.f, aux_dot_pow = 0.f;
  float* end_state = nullptr;
  int64_t end_ld = 0, end_bstride = 0;
};

// A matrix operand in global memory: element (b, row, col) of its storage order at
// ptr + b*bstride + row*ld + col, with `inner` = extent of col and `rows` = extent of row.
struct Operand {
  const void* ptr;
  int64_t ld, bstride;
  int64_t inner, rows;
  int dtype;
  bool mn_major;  // storage order is [k][m] (resp. [k][n]) rather than [m][k]
};

struct TileCoord {
  int b, mb, nb, k_begin, k_end;
};

__host__ __device__ inline int nlower_tiles_in_row(int mb, int BM, int BN, int n_blocks) {
  int c = ((mb + 1) * BM - 1) / BN + 1;
  return c < n_blocks ? c : n_blocks;
}

// Map a linear tile index to (batch, row block, column block, k range). Normally the tiles of one
// batch row are consecutive (L2 locality; under CAUSAL_KLOWER the longest row blocks first). With
// s.balanced (causal k ranges only) the index runs over work levels first (the row blocks with the
// longest k range first), then batch rows, then column blocks: decreasing work (schedule_tile).
template <int BM, int BN>
__device__ __forceinline__ TileCoord decode_tile(int t, const GemmShape& s, int m_blocks, int n_blocks,
                                                 int tiles_per_batch) {
  TileCoord c;
  c.b = t / tiles_per_batch;
  int i = t - c.b * tiles_per_batch;
  if (s.causal == CAUSAL_NLOWER) {
    int mb = 0;
    for (;;) {
      const int cnt = nlower_tiles_in_row(mb, BM, BN, n_blocks);
      if (i < cnt) break;
      i -= cnt;
      ++mb;
    }
    c.mb = mb;
    c.nb = i;
  } else if (s.balanced) {
    const int per_level = s.batches * n_blocks;
    const int level = t / per_level;
    const int rem = t - level * per_level;
    c.b = rem / n_blocks;
    c.nb = rem - c.b * n_blocks;
    c.mb = s.causal == CAUSAL_KLOWER ? m_blocks - 1 - level : level;
  } else {
    c.mb = i / n_blocks;
    c.nb = i - c.mb * n_blocks;
    if (s.causal == CAUSAL_KLOWER) c.mb = m_blocks - 1 - c.mb;
  }
  c.k_begin = 0;
  c.k_end = s.K;
  if (s.causal == CAUSAL_KLOWER) c.k_end = min(s.K, (c.mb + 1) * BM);
  if (s.causal == CAUSAL_KUPPER) c.k_begin = min(s.K, c.mb * BM);
  if (s.ksplit > 1) {
    const int kc = ksplit_chunk(s.K, s.ksplit);
    c.k_begin = min(s.K, c.b * kc);
    c.k_end = min(s.K, c.k_begin + kc);
  }
  return c;
}

inline int tiles_per_batch_host(const GemmShape& s, int BM, int BN, int m_blocks, int n_blocks) {
  if (s.causal != CAUSAL_NLOWER) return m_blocks * n_blocks;
  int n = 0;
  for (int mb = 0; mb < m_blocks; ++mb) n += nlower_tiles_in_row(mb, BM, BN, n_blocks);
  return n;
}

// Entries of tile_partial an EPI_DECAY_DG launch over (batches, T x T) may write, for every back
// end: 16 per 256 x 256 tile on CTA pairs, 8 per 128-row tile on single CTAs (columns of 128 or
// 256), 4 per 64 x 64 tile of the FMA kernel.
inline int64_t tile_partials_2d(int64_t batches, int64_t M, int64_t N) {
  auto b = [](int64_t n, int64_t t) { return (n + t - 1) / t; };
  int64_t e = 4 * b(M, 64) * b(N, 64);
  e = e > 8 * b(M, 128) * b(N, 128) ? e : 8 * b(M, 128) * b(N, 128);
  e = e > 16 * b(M, 256) * b(N, 256) ? e : 16 * b(M, 256) * b(N, 256);
  return batches * e;
}

inline int64_t decay_dg_partials(int64_t batches, int64_t T) { return tile_partials_2d(batches, T, T); }

// Entries of tile_partial a carry product with an aux dot over (batches, M x N) states may write.
inline int64_t carry_dot_partials(int64_t batches, int64_t M, int64_t N) { return tile_partials_2d(batches, M, N); }

// Host entry: validates, picks the back end from the operand types, launches on `stream`.
int run_gemm(const Operand& A, const Operand& B, const GemmShape& s, const GemmEpilogue& e, cudaStream_t stream);

// C = A B^T (over A's k range) + A2 B2^T (over K2), one accumulator: the second pair has the first
// pair's element type and storage orders; a member with batch stride 0 is shared by all batch rows.
int run_gemm2(const Operand& A, const Operand& B, const Operand* A2, const Operand* B2, const GemmShape& s,
              const GemmEpilogue& e, cudaStream_t stream);

}  // namespace ulm
