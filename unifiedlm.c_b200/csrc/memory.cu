// The fast-memory operator (the reference's kernel.py:199-238) built from the batched GEMM engine
// and the statistics scans, plus the library-level C ABI glue.
//
// Forward, per batch row (lam = exp(g), k = shift(r), D[t,s] = lam^(t-s) for s <= t):
//   stats            q = r / (w + D k),  plus operand copies qop, kop
//   scores           P = D * (qop kop^T)                     (B,T,T), tiles on/below the diagonal
//   read             fast = P vop                             causal k range
// Backward, with do = dfast:
//   scores           dS = D * (do vop^T)
//   reads            dqf = dS kop,  dk = dS^T qop,  dv = P^T do
//   stats backward   dr, dw, dg (reverse scan, deterministic reductions)
//
// The reference carries a (K x V) state between 64-token chunks and materialises it for every chunk
// (kernel.py:23-48). At the shapes this library targets (T up to a few thousand, K = slots up to
// 2048, V = dim up to 768) the T x T score matrix is far smaller than the per-chunk states and the
// whole-sequence products are fewer flops: forward T(M+D) per token against 4MD + 2C(M+D) for the
// chunked form. Results are the same function; only the summation order differs.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "gemm.cuh"

namespace ulm {

static thread_local char g_error_msg[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error_msg, sizeof(g_error_msg), fmt, ap);
  va_end(ap);
}

int current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}

int sm_count(int device) {
  static int cache[64] = {};
  if (device < 0 || device >= 64) return 148;
  if (cache[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 148;
    cache[device] = n;
  }
  return cache[device];
}

namespace {

struct SideStreams {
  std::mutex mu;
  cudaStream_t stream[64] = {};
  cudaEvent_t event[64] = {};
};

SideStreams& side_streams() {
  static SideStreams s;
  return s;
}

}  // namespace

static int g_pdl = 1;

int pdl_enabled() { return g_pdl; }

int side_stream(cudaStream_t* out) {
  const int dev = current_device();
  ULM_REQUIRE(dev >= 0 && dev < 64, "no current CUDA device (or ordinal >= 64)");
  SideStreams& ss = side_streams();
  std::lock_guard<std::mutex> lock(ss.mu);
  if (!ss.stream[dev]) {
    ULM_CUDA_TRY(cudaStreamCreateWithFlags(&ss.stream[dev], cudaStreamNonBlocking));
    ULM_CUDA_TRY(cudaEventCreateWithFlags(&ss.event[dev], cudaEventDisableTiming));
  }
  *out = ss.stream[dev];
  return ULM_OK;
}

int stream_after(cudaStream_t to, cudaStream_t from) {
  const int dev = current_device();
  ULM_REQUIRE(dev >= 0 && dev < 64, "no current CUDA device (or ordinal >= 64)");
  SideStreams& ss = side_streams();
  std::lock_guard<std::mutex> lock(ss.mu);  // one event per device: record and wait as one step
  ULM_REQUIRE(ss.event[dev] != nullptr, "stream_after before side_stream on this device");
  ULM_CUDA_TRY(cudaEventRecord(ss.event[dev], from));
  ULM_CUDA_TRY(cudaStreamWaitEvent(to, ss.event[dev], 0));
  return ULM_OK;
}

namespace {

int elem_size(int dtype) { return dtype == ULM_BF16 ? 2 : 4; }

int op_dtype_of(int prec) { return prec == ULM_PREC_FP32 ? ULM_F32 : ULM_BF16; }

GemmEpilogue make_epilogue(int kind, int out_dtype, void* out, int64_t ldo, int64_t bstride, const float* g) {
  GemmEpilogue e;
  e.kind = kind;
  e.out_dtype = out_dtype;
  e.out = out;
  e.ldo = ldo;
  e.out_bstride = bstride;
  e.g = g;
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

// elementwise copy with type conversion between row strides (fp32/bf16 -> fp32/bf16)
__global__ void convert_rows_kernel(const void* __restrict__ src, int src_dtype, int64_t lds, void* __restrict__ dst,
                                    int dst_dtype, int64_t ldd, int64_t rows, int64_t cols) {
  const int64_t n = rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t rr = i / cols, cc = i - rr * cols;
    const float v = src_dtype == ULM_F32 ? static_cast<const float*>(src)[rr * lds + cc]
                                         : __bfloat162float(static_cast<const __nv_bfloat16*>(src)[rr * lds + cc]);
    if (dst_dtype == ULM_F32)
      static_cast<float*>(dst)[rr * ldd + cc] = v;
    else
      static_cast<__nv_bfloat16*>(dst)[rr * ldd + cc] = __float2bfloat16_rn(v);
  }
}

// 8 consecutive elements per thread with 16-byte loads and stores
__global__ void convert_rows_vec8_kernel(const void* __restrict__ src, int src_dtype, int64_t lds,
                                         void* __restrict__ dst, int dst_dtype, int64_t ldd, int64_t rows,
                                         int64_t cols8) {
  pdl_enter();
  const int64_t n = rows * cols8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t rr = i / cols8, cc = (i - rr * cols8) * 8;
    float v[8];
    if (src_dtype == ULM_F32) {
      const float4* s4 = reinterpret_cast<const float4*>(static_cast<const float*>(src) + rr * lds + cc);
      const float4 a = s4[0], b = s4[1];
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
      const uint4 pk = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(src) + rr * lds + cc);
      const uint32_t w4[4] = {pk.x, pk.y, pk.z, pk.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 h;
        memcpy(&h, &w4[j], 4);
        const float2 f = __bfloat1622float2(h);
        v[2 * j] = f.x;
        v[2 * j + 1] = f.y;
      }
    }
    if (dst_dtype == ULM_F32) {
      float4* d4 = reinterpret_cast<float4*>(static_cast<float*>(dst) + rr * ldd + cc);
      d4[0] = make_float4(v[0], v[1], v[2], v[3]);
      d4[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
      uint4 pk;
      uint32_t w4[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        memcpy(&w4[j], &h, 4);
      }
      pk.x = w4[0]; pk.y = w4[1]; pk.z = w4[2]; pk.w = w4[3];
      *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(dst) + rr * ldd + cc) = pk;
    }
  }
}

int convert_rows(const void* src, int sdt, int64_t lds, void* dst, int ddt, int64_t ldd, int64_t rows, int64_t cols,
                 cudaStream_t st) {
  if (rows * cols == 0) return ULM_OK;
  if (src == dst && sdt == ddt && lds == ldd) return ULM_OK;  // the caller passed the array as its own copy
  if (cols % 8 == 0 && lds % 8 == 0 && ldd % 8 == 0 && is_aligned16(src) && is_aligned16(dst)) {
    const int64_t blocks = cdiv(rows * (cols / 8), 256);
    const unsigned grid = (unsigned)(blocks < 16 * 148 ? blocks : 16 * 148);
    return launch_pdl(convert_rows_vec8_kernel, dim3(grid), dim3(256), 0, st, src, sdt, lds, dst, ddt, ldd, rows,
                      cols / 8);
  }
  const int64_t blocks = cdiv(rows * cols, 256);
  const unsigned grid = (unsigned)(blocks < 8 * 148 ? blocks : 8 * 148);
  convert_rows_kernel<<<grid, 256, 0, st>>>(src, sdt, lds, dst, ddt, ldd, rows, cols);
  ULM_LAUNCH_CHECK("convert_rows_kernel");
  return ULM_OK;
}

// wmu[m][d] = w[m] * mu[d][m] (the combine's weight as the second B operand of the read product,
// MN-major over d) in the operand type, rows padded to ld
__global__ void combine_weight_t_kernel(const float* __restrict__ mu, const float* __restrict__ w,
                                        void* __restrict__ out, int dt, int64_t ld, int D, int M) {
  __shared__ float tile[32][33];
  const int m0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
  for (int i = ty; i < 32; i += 8) {
    const int d = d0 + i, m = m0 + tx;
    tile[i][tx] = (d < D && m < M) ? mu[(int64_t)d * M + m] * w[m] : 0.f;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int m = m0 + i, d = d0 + tx;
    if (m < M && d < D) {
      const float v = tile[tx][i];
      if (dt == ULM_F32)
        static_cast<float*>(out)[(int64_t)m * ld + d] = v;
      else
        static_cast<__nv_bfloat16*>(out)[(int64_t)m * ld + d] = __float2bfloat16_rn(v);
    }
  }
}

// mw[d][m] = mu[d][m] * w[m] (the combine's weight as the second B operand of the dq product,
// MN-major over m) in the operand type, rows padded to ld
__global__ void combine_weight_kernel(const float* __restrict__ mu, const float* __restrict__ w,
                                      void* __restrict__ out, int dt, int64_t ld, int D, int M) {
  const int64_t n = (int64_t)D * M;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t d = i / M, m = i - d * M;
    const float v = mu[i] * w[m];
    if (dt == ULM_F32)
      static_cast<float*>(out)[d * ld + m] = v;
    else
      static_cast<__nv_bfloat16*>(out)[d * ld + m] = __float2bfloat16_rn(v);
  }
}

// The combine's parameter gradients from the split-K partials of G = dy^T q (S x D x M): a CTA takes
// 32 slots x 32 rows (threads: 32 slots x 8 row groups), writes dmu[d][m] = w[m] G[d][m] and one
// partial of sum_d mu[d][m] G[d][m] per slot, partials and rows added in a fixed order.
constexpr int COMBINE_ROWS = 32;
__global__ void __launch_bounds__(256)
    combine_grad_kernel(const float* __restrict__ gpart, int S, const float* __restrict__ mu,
                        const float* __restrict__ w, float* __restrict__ dmu, float* __restrict__ dw_part, int D,
                        int M) {
  __shared__ float red[8][32];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int m = blockIdx.x * 32 + tx;
  const int d0 = blockIdx.y * COMBINE_ROWS;
  float acc = 0.f;
  if (m < M) {
    const float wm = w[m];
    for (int d = d0 + ty; d < min(D, d0 + COMBINE_ROWS); d += 8) {
      const int64_t i = (int64_t)d * M + m;
      float gsum = 0.f;
      for (int sp = 0; sp < S; ++sp) gsum += gpart[(int64_t)sp * D * M + i];
      dmu[i] = gsum * wm;
      acc = fmaf(mu[i], gsum, acc);
    }
  }
  red[ty][tx] = acc;
  __syncthreads();
  if (ty == 0 && m < M) {
    float t = red[0][tx];
    for (int j = 1; j < 8; ++j) t += red[j][tx];
    dw_part[(int64_t)blockIdx.y * M + m] = t;
  }
}

// out[i] += sum over p of part[p][i], in order
__global__ void add_parts_kernel(const float* __restrict__ part, int nparts, int64_t n, float* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float t = 0.f;
  for (int p = 0; p < nparts; ++p) t += part[(int64_t)p * n + i];
  out[i] += t;
}

int check_prec(int prec) {
  ULM_REQUIRE(prec == ULM_PREC_BF16 || prec == ULM_PREC_FP32, "prec must be ULM_PREC_BF16 or ULM_PREC_FP32");
  return ULM_OK;
}

// The block's learned scalars from their log parameters (model.py:72, 75, 84), in fp32 as PyTorch
// evaluates the same expressions: w = exp(clamp(log_w, -7, 12)), eps = exp(clamp(log_eps, -10, 10)),
// g = -exp(log_rate). Thread 0 of block 0 also writes the two scalars.
__global__ void block_scalars_fwd_kernel(const float* __restrict__ log_w, const float* __restrict__ log_eps,
                                         const float* __restrict__ log_rate, float* __restrict__ w,
                                         float* __restrict__ eps, float* __restrict__ g, int64_t M) {
  pdl_enter();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < M) w[i] = expf(fminf(fmaxf(log_w[i], -7.f), 12.f));
  if (i == 0) {
    *eps = expf(fminf(fmaxf(*log_eps, -10.f), 10.f));
    *g = -expf(*log_rate);
  }
}

// Their backward, as PyTorch's autograd of the same expressions computes it: exp passes
// grad * exp(x), clamp passes the gradient where min <= x <= max and zero elsewhere, negation
// flips the sign (so dlog_rate = -(dg * exp(log_rate)) = dg * g).
__global__ void block_scalars_bwd_kernel(const float* __restrict__ log_w, const float* __restrict__ log_eps,
                                         const float* __restrict__ w, const float* __restrict__ eps,
                                         const float* __restrict__ g, const float* __restrict__ dw,
                                         const float* __restrict__ deps, const float* __restrict__ dg,
                                         float* __restrict__ dlog_w, float* __restrict__ dlog_eps,
                                         float* __restrict__ dlog_rate, int64_t M) {
  pdl_enter();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < M) {
    const float x = log_w[i];
    dlog_w[i] = (x >= -7.f && x <= 12.f) ? dw[i] * w[i] : 0.f;
  }
  if (i == 0) {
    const float x = *log_eps;
    *dlog_eps = (x >= -10.f && x <= 10.f) ? (*deps) * (*eps) : 0.f;
    *dlog_rate = (*dg) * (*g);
  }
}

}  // namespace

}  // namespace ulm

using namespace ulm;

extern "C" int ulm_block_scalars_fwd(const float* log_w, const float* log_eps, const float* log_rate, float* w,
                                     float* eps, float* g, int64_t M, void* stream) {
  ULM_REQUIRE(M >= 0 && M < (1ll << 31), "bad extent M=%lld", (long long)M);
  ULM_REQUIRE(log_eps && log_rate && eps && g && (M == 0 || (log_w && w)), "null pointer argument");
  const unsigned grid = (unsigned)(M > 0 ? cdiv(M, 256) : 1);
  return launch_pdl(block_scalars_fwd_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream), log_w,
                    log_eps, log_rate, w, eps, g, M);
}

extern "C" int ulm_block_scalars_bwd(const float* log_w, const float* log_eps, const float* w, const float* eps,
                                     const float* g, const float* dw, const float* deps, const float* dg,
                                     float* dlog_w, float* dlog_eps, float* dlog_rate, int64_t M, void* stream) {
  ULM_REQUIRE(M >= 0 && M < (1ll << 31), "bad extent M=%lld", (long long)M);
  ULM_REQUIRE(log_eps && eps && g && deps && dg && dlog_eps && dlog_rate && (M == 0 || (log_w && w && dw && dlog_w)),
              "null pointer argument");
  const unsigned grid = (unsigned)(M > 0 ? cdiv(M, 256) : 1);
  return launch_pdl(block_scalars_bwd_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream), log_w,
                    log_eps, w, eps, g, dw, deps, dg, dlog_w, dlog_eps, dlog_rate, M);
}

extern "C" const char* ulm_last_error(void) { return g_error_msg; }

extern "C" int ulm_version(void) { return 1; }

extern "C" int ulm_device_error(int* site) {
  ULM_REQUIRE(site, "null site pointer");
  ULM_CUDA_TRY(cudaDeviceSynchronize());
  int v = 0;
  ULM_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)));
  const int zero = 0;
  ULM_CUDA_TRY(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)));
  *site = v;
  return ULM_OK;
}

extern "C" int64_t ulm_operand_ld(int64_t n) { return ((n + 7) / 8) * 8; }

extern "C" int ulm_set_gemm_pairs(int enable) {
  const int old = g_gemm_pairs;
  g_gemm_pairs = enable ? 1 : 0;
  return old;
}

extern "C" int ulm_set_pdl(int enable) {
  const int old = g_pdl;
  g_pdl = enable ? 1 : 0;
  return old;
}

extern "C" int ulm_set_epilogue_mode(int mode) {
  if (mode < EPI_MODE_DIRECT || mode > EPI_MODE_WARP) return -1;
  const int old = g_epi_mode;
  g_epi_mode = mode;
  return old;
}

extern "C" int ulm_decayed_scores(const void* a, int64_t lda, const void* bb, int64_t ldb, void* P, int64_t ldp,
                                  const float* g, int64_t B, int64_t T, int64_t K, int prec, void* stream) {
  if (int rc = check_prec(prec)) return rc;
  ULM_REQUIRE(B >= 0 && T >= 0 && K >= 0, "negative extent");
  ULM_REQUIRE(T < (1 << 30) && K < (1 << 30) && B < (1 << 30), "extent too large");
  ULM_REQUIRE(lda >= K && ldb >= K && ldp >= T, "row stride shorter than the row");
  const int dt = op_dtype_of(prec);
  Operand A{a, lda, T * lda, K, T, dt, false};
  Operand Bo{bb, ldb, T * ldb, K, T, dt, false};
  GemmShape s{(int)B, (int)T, (int)T, (int)K, CAUSAL_NLOWER};
  GemmEpilogue e = make_epilogue(EPI_DECAY, dt, P, ldp, T * ldp, g);
  return run_gemm(A, Bo, s, e, static_cast<cudaStream_t>(stream));
}

extern "C" int ulm_causal_apply(const void* P, int64_t ldp, const void* c, int64_t ldc, void* o, int64_t ldo,
                                int o_dtype, int transpose, int64_t B, int64_t T, int64_t V, int prec, void* stream) {
  if (int rc = check_prec(prec)) return rc;
  ULM_REQUIRE(B >= 0 && T >= 0 && V >= 0, "negative extent");
  ULM_REQUIRE(T < (1 << 30) && V < (1 << 30) && B < (1 << 30), "extent too large");
  ULM_REQUIRE(ldp >= T && ldc >= V && ldo >= V, "row stride shorter than the row");
  ULM_REQUIRE(o_dtype == ULM_F32 || o_dtype == ULM_BF16, "bad o_dtype");
  const int dt = op_dtype_of(prec);
  // forward : o[t][v] = sum_s P[t][s] c[s][v]  -> A = P (K-major), B = c ([k=s][n=v], MN-major)
  // reversed: o[s][v] = sum_t P[t][s] c[t][v]  -> A = P read as [k=t][m=s] (MN-major)
  Operand A{P, ldp, T * ldp, T, T, dt, transpose != 0};
  Operand Bo{c, ldc, T * ldc, V, T, dt, true};
  GemmShape s{(int)B, (int)T, (int)V, (int)T, transpose ? CAUSAL_KUPPER : CAUSAL_KLOWER};
  GemmEpilogue e = make_epilogue(EPI_STORE, o_dtype, o, ldo, T * ldo, nullptr);
  return run_gemm(A, Bo, s, e, static_cast<cudaStream_t>(stream));
}

// ---- the chunk-carry form of the fast read (long sequences) ----------------------------------
// For T well above the slot and value widths the whole-sequence products cost T (M + D) flops per
// token; the reference's chunked form costs 4 M D + 2 C (M + D). Here the chunked form runs on the
// same GEMM engine: a carry product walks the chunks with the (M x D) state in the tensor cores'
// accumulator (written once per chunk boundary, in the operand type), the inter-chunk read is a
// product against those states with a per-row decay, and the intra-chunk part is the
// whole-sequence machinery on C-long pieces (batches B * T / C). The backward runs one reverse
// carry (the state of q dO^T from the chunks to the right), three inter-chunk products and the
// intra-chunk products; d/dg gets three extra position-weighted sums (see chunk_read_bwd).
namespace ulm {
namespace {

// -1: automatic; 0: always the whole-sequence form; > 0: this chunk length wherever T is a multiple
// of it with at least two chunks (ulm_set_chunk_mode)
int g_chunk_mode = -1;

constexpr int DOT_BLOCKS = 296;  // fixed grid of the weighted dot products (deterministic partials)

// Chunk length of the operator's fast read, 0 = the whole-sequence form. Automatic: on the tensor
// cores the largest C in {1024, 512, 256} (multiples of the pair tiles' 256 rows) that divides T into
// at least two chunks, in fp32 C = 64 (the FMA back end's 64-row tiles), used where the
// whole-sequence form's flops per token T (M + D) exceed 1.25 x the chunked form's
// 4 M D + 2 C (M + D) (the margin pays for the chunked form's extra passes: the per-row decays,
// the state writes and reads). Measured on B200, bf16, 65536 tokens per call: the chunked form with
// C = 1024 is 15-16% faster at T = 8192 at D 512 / M 1024 and at D 768 / M 2048, 6% slower at
// T = 4096 (42M widths) and slower still below; C = 1024 beat 512 and 256 at every T, since fewer
// chunk boundaries mean fewer state writes and reads.
int chunk_len(int64_t T, int64_t M, int64_t D, int prec) {
  if (g_chunk_mode == 0 || M == 0 || D == 0) return 0;
  auto fits = [&](int64_t C) { return T % C == 0 && T / C >= 2; };
  if (g_chunk_mode > 0) return fits(g_chunk_mode) ? g_chunk_mode : 0;
  int64_t C = 0;
  if (prec == ULM_PREC_FP32) {
    C = fits(64) ? 64 : 0;
  } else {
    for (int64_t c : {1024, 512, 256})
      if (!C && fits(c)) C = c;
  }
  if (!C) return 0;
  const double whole = (double)T * (double)(M + D);
  const double chunked = 4.0 * (double)M * (double)D + 2.0 * (double)C * (double)(M + D);
  return whole > 1.25 * chunked ? (int)C : 0;
}

struct ChunkFwdLayout {
  void* Pc;    // (B, T, C) intra-chunk decayed scores, operand type
  void* Hs;    // (B, NT, M, ldD) state entering each chunk (slot 0 = zero), operand type
  float* Fi;   // (B, T, D) inter-chunk read, fp32
  void* work;  // the carry's decayed values (B, T, ldD), then the intra read's addend (B, T, D)
  int64_t bytes;
};

ChunkFwdLayout chunk_fwd_layout(void* base, int64_t B, int64_t T, int64_t M, int64_t D, int64_t C, int prec) {
  const int64_t es = prec == ULM_PREC_FP32 ? 4 : 2, ldd = ulm_operand_ld(D), NT = T / C;
  uint8_t* p = static_cast<uint8_t*>(base);
  ChunkFwdLayout L;
  int64_t off = 0;
  L.Pc = p + off;
  off += align256(B * T * C * es);
  L.Hs = p + off;
  off += align256(B * NT * M * ldd * es);
  L.Fi = reinterpret_cast<float*>(p + off);
  off += align256(B * T * D * 4);
  L.work = p + off;
  off += align256(B * T * std::max<int64_t>(ldd * es, D * 4));
  L.bytes = off;
  return L;
}

struct ChunkBwdLayout {
  void* dSc;      // (B, T, C) intra-chunk score gradient
  void* Rs;       // (B, NT, M, ldD) reverse states (slot NT-1 = zero)
  float* Fv;      // (B, T, D) inter-chunk part of dv, fp32
  void* dOhat;    // (B, T, ldD) upstream gradient times lam^(position in chunk)
  void* auxv;     // (B, T, D) the intra dv product's addend in dv's type
  float* tiles;   // d/dg partials: score epilogue, reverse-carry dot, the two weighted sums
  int64_t n_score, n_carry, n_tiles;
  int64_t bytes;
};

ChunkBwdLayout chunk_bwd_layout(void* base, int64_t B, int64_t T, int64_t M, int64_t D, int64_t C, int prec) {
  const int64_t es = prec == ULM_PREC_FP32 ? 4 : 2, ldd = ulm_operand_ld(D), NT = T / C;
  uint8_t* p = static_cast<uint8_t*>(base);
  ChunkBwdLayout L;
  int64_t off = 0;
  L.dSc = p + off;
  off += align256(B * T * C * es);
  L.Rs = p + off;
  off += align256(B * NT * M * ldd * es);
  L.Fv = reinterpret_cast<float*>(p + off);
  off += align256(B * T * D * 4);
  L.dOhat = p + off;
  off += align256(B * T * ldd * es);
  L.auxv = p + off;
  off += align256(B * T * D * 4);
  L.n_score = decay_dg_partials(B * NT, C);
  L.n_carry = carry_dot_partials(B, M, D);
  L.n_tiles = L.n_score + L.n_carry + 2 * DOT_BLOCKS;
  L.tiles = reinterpret_cast<float*>(p + off);
  off += align256(L.n_tiles * 4);
  L.bytes = off;
  return L;
}

// dst[r][d] = lam^(a + s * (r mod C)) * src[r][d] for d < D over `rows` rows of stride ld (the row's
// position inside its chunk is r mod C because T is a multiple of C); one warp per row, the factor
// computed once per row, the columns strided over the lanes
template <typename E>
__global__ void __launch_bounds__(256)
    chunk_scale_rows_kernel(const E* __restrict__ src, E* __restrict__ dst, int64_t ld, int64_t rows, int D, int C,
                            const float* __restrict__ g, float a, float s) {
  pdl_enter();
  const float gl = *g;
  const int lane = threadIdx.x & 31;
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += nw) {
    const float f = expf(gl * (a + s * (float)(int)(r % C)));
    const E* sr = src + r * ld;
    E* dr = dst + r * ld;
    for (int d = lane; d < D; d += 32) {
      if constexpr (sizeof(E) == 4)
        dr[d] = sr[d] * f;
      else
        dr[d] = __float2bfloat16_rn(__bfloat162float(sr[d]) * f);
    }
  }
}

int chunk_scale_rows(const void* src, void* dst, int dt, int64_t ld, int64_t rows, int64_t D, int C, const float* g,
                     float a, float s, cudaStream_t st) {
  if (rows * D == 0) return ULM_OK;
  const unsigned grid = (unsigned)std::min<int64_t>(cdiv(rows, 8), 16 * 148);
  if (dt == ULM_F32)
    return launch_pdl(chunk_scale_rows_kernel<float>, dim3(grid), dim3(256), 0, st, static_cast<const float*>(src),
                      static_cast<float*>(dst), ld, rows, (int)D, C, g, a, s);
  return launch_pdl(chunk_scale_rows_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, st,
                    static_cast<const __nv_bfloat16*>(src), static_cast<__nv_bfloat16*>(dst), ld, rows, (int)D, C, g,
                    a, s);
}

// out[i] = x[i] + f[i] in x's type (the combine's residual plus the inter-chunk read)
__global__ void add_rows_kernel(const void* __restrict__ x, int xdt, const float* __restrict__ f, void* __restrict__ out,
                                int64_t n) {
  pdl_enter();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    if (xdt == ULM_F32)
      static_cast<float*>(out)[i] = static_cast<const float*>(x)[i] + f[i];
    else
      static_cast<__nv_bfloat16*>(out)[i] =
          __float2bfloat16_rn(__bfloat162float(static_cast<const __nv_bfloat16*>(x)[i]) + f[i]);
  }
}

// part[blockIdx.x] = sum over rows r < rows, d < D of (wa + ws * (r mod C)) * x[r][d] * y[r][d]
// (x in its type with row stride ldx, y fp32 with row stride D); DOT_BLOCKS blocks of 8 warps, one
// warp per row at a time, fixed order
__global__ void __launch_bounds__(256)
    weighted_dot_kernel(const void* __restrict__ x, int xdt, int64_t ldx, const float* __restrict__ y, int64_t rows,
                        int D, int C, float wa, float ws, float* __restrict__ part) {
  pdl_enter();
  __shared__ float red[8];
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  float acc = 0.f;
  for (int64_t r = (int64_t)blockIdx.x * 8 + wp; r < rows; r += (int64_t)gridDim.x * 8) {
    const float wgt = wa + ws * (float)(int)(r % C);
    const float* yr = y + r * D;
    float row = 0.f;
    if (xdt == ULM_F32) {
      const float* xr = static_cast<const float*>(x) + r * ldx;
      for (int d = lane; d < D; d += 32) row = fmaf(xr[d], yr[d], row);
    } else {
      const __nv_bfloat16* xr = static_cast<const __nv_bfloat16*>(x) + r * ldx;
      for (int d = lane; d < D; d += 32) row = fmaf(__bfloat162float(xr[d]), yr[d], row);
    }
    acc = fmaf(wgt, row, acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) red[wp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < 8; ++i) t += red[i];
    part[blockIdx.x] = t;
  }
}

// Forward fast read in the chunk-carry form: out = P v + lam^(i+1) q H (+ x + q wmu^T with the
// combine's x and wmu), from the operand copies; `saved` (chunk_fwd_layout) keeps what the backward
// reads. end_state (optional, fp32 (B, M, D)): the state after the last position,
// sum_s lam^(T-1-s) k_s v_s^T.
int chunk_read_fwd(const void* qop, const void* kop, const void* vop, const float* g, void* saved, void* out,
                   int out_dtype, const void* x, const void* wmu, float* end_state, int64_t B, int64_t T, int64_t M,
                   int64_t D, int C, int prec, cudaStream_t st) {
  const int dt = op_dtype_of(prec);
  const int64_t es = elem_size(dt), ldm = ulm_operand_ld(M), ldd = ulm_operand_ld(D), NT = T / C;
  ChunkFwdLayout L = chunk_fwd_layout(saved, B, T, M, D, C, prec);
  // the carry's values: v_s lam^(C-1-j), j the position in its chunk
  if (int rc = chunk_scale_rows(vop, L.work, dt, ldd, B * T, D, C, g, (float)(C - 1), -1.f, st)) return rc;
  // slot 0 of every batch row: the zero state entering the first chunk
  ULM_CUDA_TRY(cudaMemset2DAsync(L.Hs, (size_t)(NT * M * ldd * es), 0, (size_t)(M * ldd * es), (size_t)B, st));
  {
    // H_{n+1} = lam^C H_n + k_n^T vhat_n  (A = k as [pos][slot], B = vhat as [pos][d])
    Operand A{kop, ldm, T * ldm, M, T, dt, true};
    Operand Bv{L.work, ldd, T * ldd, D, T, dt, true};
    GemmShape s{(int)B, (int)M, (int)D, (int)T, CAUSAL_NONE};
    s.carry = CARRY_FWD;
    s.carry_C = C;
    s.carry_chunks = (int)NT;
    s.carry_end = end_state ? 1 : 0;
    GemmEpilogue e = make_epilogue(EPI_STORE, dt, L.Hs, ldd, M * ldd, g);
    e.end_state = end_state;
    e.end_ld = D;
    e.end_bstride = M * D;
    if (int rc = run_gemm(A, Bv, s, e, st)) return rc;
  }
  {
    // inter-chunk read F = lam^(i+1) q H_n, batches (b, n)
    Operand Aq{qop, ldm, C * ldm, M, C, dt, false};
    Operand Bh{L.Hs, ldd, M * ldd, D, M, dt, true};
    GemmShape s{(int)(B * NT), C, (int)D, (int)M, CAUSAL_NONE};
    GemmEpilogue e = make_epilogue(EPI_ROW_DECAY, ULM_F32, L.Fi, D, C * D, g);
    e.rd_a = 1.f;
    e.rd_s = 1.f;
    if (int rc = run_gemm(Aq, Bh, s, e, st)) return rc;
  }
  if (int rc = ulm_decayed_scores(qop, ldm, kop, ldm, L.Pc, C, g, B * NT, C, M, prec, st)) return rc;
  // the intra read's addend in the output's type: F, plus x for the combine
  const void* addend = L.Fi;
  if (x) {
    const unsigned grid = (unsigned)std::min<int64_t>(cdiv(B * T * D, 256), 8 * 148);
    if (int rc = launch_pdl(add_rows_kernel, dim3(grid), dim3(256), 0, st, x, out_dtype, (const float*)L.Fi, L.work,
                            B * T * D))
      return rc;
    addend = L.work;
  } else if (out_dtype != ULM_F32) {
    if (int rc = convert_rows(L.Fi, ULM_F32, D, L.work, out_dtype, D, B * T, D, st)) return rc;
    addend = L.work;
  }
  // out = P v (+ q wmu^T) + addend, intra-chunk causal k range
  Operand Ap{L.Pc, C, (int64_t)C * C, C, C, dt, false};
  Operand Bv{vop, ldd, C * ldd, D, C, dt, true};
  GemmShape s{(int)(B * NT), C, (int)D, C, CAUSAL_KLOWER};
  GemmEpilogue e = make_epilogue(EPI_STORE_ADD, out_dtype, out, D, C * D, nullptr);
  e.aux = addend;
  e.ld_aux = D;
  e.aux_bstride = C * D;
  e.vec_ok = e.vec_ok && is_aligned16(addend);
  if (wmu) {
    Operand A2{qop, ldm, C * ldm, M, C, dt, false};
    Operand B2{wmu, ldd, 0, D, M, dt, true};
    s.K2 = (int)M;
    return run_gemm2(Ap, Bv, &A2, &B2, s, e, st);
  }
  return run_gemm(Ap, Bv, s, e, st);
}

// Backward fast read in the chunk-carry form, for dO (doop, the operand copy of dfast or dy):
//   dq = dS k + lam^(i+1) dO H_n^T (+ dy mw with the combine's mw)
//   dk = dS^T q + lam^(C-j) v R_n^T,  dv = P^T dO + lam^(C-j) k R_n
// with dS the intra-chunk score gradient and R_n = sum_{t past chunk n} lam^(t - start of chunk
// n+1) q_t dO_t^T (the reverse carry). d/dg of the fast read in tile partials (layout in L): the
// score epilogue's sum (t-s) P dP inside chunks, plus across chunks
//   sum_t (i+1) dO_t . F_t  +  C lam^(C+1) sum_n <R_n, H_n>  +  sum_s (C-1-j) v_s . dv_inter_s,
// the derivative of the lam^(i+1) read factor, of the lam^C carry and of the lam^(C-1-j) write
// factor. dq and dk are fp32 (B,T,M); dv in dv_dtype.
int chunk_read_bwd(const void* doop, const void* qop, const void* kop, const void* vop, const float* g,
                   const void* saved, void* work, float* dqf, float* dk, void* dv, int dv_dtype, const void* mw,
                   int64_t B, int64_t T, int64_t M, int64_t D, int C, int prec, cudaStream_t st, cudaStream_t side,
                   ChunkBwdLayout* out_layout) {
  const int dt = op_dtype_of(prec);
  const int64_t es = elem_size(dt), ldm = ulm_operand_ld(M), ldd = ulm_operand_ld(D), NT = T / C;
  ChunkFwdLayout F = chunk_fwd_layout(const_cast<void*>(saved), B, T, M, D, C, prec);
  ChunkBwdLayout L = chunk_bwd_layout(work, B, T, M, D, C, prec);
  *out_layout = L;
  ULM_CUDA_TRY(cudaMemsetAsync(L.tiles, 0, L.n_tiles * sizeof(float), st));
  if (int rc = chunk_scale_rows(doop, L.dOhat, dt, ldd, B * T, D, C, g, 0.f, 1.f, st)) return rc;
  ULM_CUDA_TRY(cudaMemset2DAsync(static_cast<uint8_t*>(L.Rs) + (NT - 1) * M * ldd * es, (size_t)(NT * M * ldd * es), 0,
                                 (size_t)(M * ldd * es), (size_t)B, st));
  float* t_score = L.tiles;
  float* t_carry = t_score + L.n_score;
  float* t_readA = t_carry + L.n_carry;
  float* t_writeC = t_readA + DOT_BLOCKS;
  const unsigned dgrid = DOT_BLOCKS;
  if (int rc = stream_after(side, st)) return rc;
  // ---- side stream: reverse carry and the inter-chunk dk / dv ----
  {
    // R_{n-1} = lam^C R_n + q_n^T dOhat_n for n = NT-1 .. 1, with C lam^(C+1) <R_n, H_n> summed
    Operand A{qop, ldm, T * ldm, M, T, dt, true};
    Operand Bo{L.dOhat, ldd, T * ldd, D, T, dt, true};
    GemmShape s{(int)B, (int)M, (int)D, (int)T, CAUSAL_NONE};
    s.carry = CARRY_REV;
    s.carry_C = C;
    s.carry_chunks = (int)NT;
    GemmEpilogue e = make_epilogue(EPI_STORE, dt, L.Rs, ldd, M * ldd, g);
    e.aux = F.Hs;
    e.ld_aux = ldd;
    e.aux_bstride = M * ldd;
    e.tile_partial = t_carry;
    e.aux_dot_scale = (float)C;
    e.aux_dot_pow = (float)(C + 1);
    e.vec_ok = e.vec_ok && is_aligned16(F.Hs);
    if (int rc = run_gemm(A, Bo, s, e, side)) return rc;
  }
  {
    // dv_inter = lam^(C-j) k_n R_n  (B = R_n read as [slot][d]: MN-major over d)
    Operand Ak{kop, ldm, C * ldm, M, C, dt, false};
    Operand Br{L.Rs, ldd, M * ldd, D, M, dt, true};
    GemmShape s{(int)(B * NT), C, (int)D, (int)M, CAUSAL_NONE};
    GemmEpilogue e = make_epilogue(EPI_ROW_DECAY, ULM_F32, L.Fv, D, C * D, g);
    e.rd_a = (float)C;
    e.rd_s = -1.f;
    if (int rc = run_gemm(Ak, Br, s, e, side)) return rc;
  }
  {
    // dk_inter = lam^(C-j) v_n R_n^T  (B = R_n as [slot][d]: K-major)
    Operand Av{vop, ldd, C * ldd, D, C, dt, false};
    Operand Br{L.Rs, ldd, M * ldd, D, M, dt, false};
    GemmShape s{(int)(B * NT), C, (int)M, (int)D, CAUSAL_NONE};
    GemmEpilogue e = make_epilogue(EPI_ROW_DECAY, ULM_F32, dk, M, C * M, g);
    e.rd_a = (float)C;
    e.rd_s = -1.f;
    if (int rc = run_gemm(Av, Br, s, e, side)) return rc;
  }
  // sum_s (C-1-j) v_s . dv_inter_s
  if (int rc = launch_pdl(weighted_dot_kernel, dim3(dgrid), dim3(256), 0, side, vop, dt, ldd, (const float*)L.Fv,
                          B * T, (int)D, C, (float)(C - 1), -1.f, t_writeC))
    return rc;
  // the intra dv product's addend in dv's type
  const void* addv = L.Fv;
  if (dv_dtype != ULM_F32) {
    if (int rc = convert_rows(L.Fv, ULM_F32, D, L.auxv, dv_dtype, D, B * T, D, side)) return rc;
    addv = L.auxv;
  }
  // ---- main stream: intra score gradient, then dq ----
  {
    Operand A{doop, ldd, C * ldd, D, C, dt, false};
    Operand Bo{vop, ldd, C * ldd, D, C, dt, false};
    GemmShape s{(int)(B * NT), C, C, (int)D, CAUSAL_NLOWER};
    GemmEpilogue e = make_epilogue(EPI_DECAY_DG, dt, L.dSc, C, (int64_t)C * C, g);
    e.aux = F.Pc;
    e.ld_aux = C;
    e.aux_bstride = (int64_t)C * C;
    e.tile_partial = t_score;
    e.vec_ok = e.vec_ok && is_aligned16(F.Pc);
    if (int rc = run_gemm(A, Bo, s, e, st)) return rc;
  }
  if (int rc = stream_after(side, st)) return rc;  // the side stream's intra products need dS
  {
    // dq_inter = lam^(i+1) dO_n H_n^T  (B = H_n as [slot][d]: K-major)
    Operand Ad{doop, ldd, C * ldd, D, C, dt, false};
    Operand Bh{F.Hs, ldd, M * ldd, D, M, dt, false};
    GemmShape s{(int)(B * NT), C, (int)M, (int)D, CAUSAL_NONE};
    GemmEpilogue e = make_epilogue(EPI_ROW_DECAY, ULM_F32, dqf, M, C * M, g);
    e.rd_a = 1.f;
    e.rd_s = 1.f;
    if (int rc = run_gemm(Ad, Bh, s, e, st)) return rc;
  }
  // sum_t (i+1) dO_t . F_t
  if (int rc = launch_pdl(weighted_dot_kernel, dim3(dgrid), dim3(256), 0, st, doop, dt, ldd, (const float*)F.Fi,
                          B * T, (int)D, C, 1.f, 1.f, t_readA))
    return rc;
  {
    // dq = dS k (+ dy mw) + dq_inter, in place
    Operand A{L.dSc, C, (int64_t)C * C, C, C, dt, false};
    Operand Bk{kop, ldm, C * ldm, M, C, dt, true};
    GemmShape s{(int)(B * NT), C, (int)M, C, CAUSAL_KLOWER};
    GemmEpilogue e = make_epilogue(EPI_STORE_ADD, ULM_F32, dqf, M, C * M, nullptr);
    e.aux = dqf;
    e.ld_aux = M;
    e.aux_bstride = C * M;
    if (mw) {
      Operand A2{doop, ldd, C * ldd, D, C, dt, false};
      Operand B2{mw, ldm, 0, M, D, dt, true};
      s.K2 = (int)D;
      if (int rc = run_gemm2(A, Bk, &A2, &B2, s, e, st)) return rc;
    } else if (int rc = run_gemm(A, Bk, s, e, st)) {
      return rc;
    }
  }
  {
    // side: dk = dS^T q + dk_inter, in place
    Operand A{L.dSc, C, (int64_t)C * C, C, C, dt, true};
    Operand Bq{qop, ldm, C * ldm, M, C, dt, true};
    GemmShape s{(int)(B * NT), C, (int)M, C, CAUSAL_KUPPER};
    GemmEpilogue e = make_epilogue(EPI_STORE_ADD, ULM_F32, dk, M, C * M, nullptr);
    e.aux = dk;
    e.ld_aux = M;
    e.aux_bstride = C * M;
    if (int rc = run_gemm(A, Bq, s, e, side)) return rc;
  }
  {
    // side: dv = P^T dO + dv_inter
    Operand A{F.Pc, C, (int64_t)C * C, C, C, dt, true};
    Operand Bo{doop, ldd, C * ldd, D, C, dt, true};
    GemmShape s{(int)(B * NT), C, (int)D, C, CAUSAL_KUPPER};
    GemmEpilogue e = make_epilogue(EPI_STORE_ADD, dv_dtype, dv, D, C * D, nullptr);
    e.aux = addv;
    e.ld_aux = D;
    e.aux_bstride = C * D;
    e.vec_ok = e.vec_ok && is_aligned16(addv);
    if (int rc = run_gemm(A, Bo, s, e, side)) return rc;
  }
  return stream_after(st, side);  // join
}

}  // namespace
}  // namespace ulm

extern "C" int ulm_set_chunk_mode(int mode) {
  if (mode < -1 || (mode > 0 && (mode % 64 != 0 || mode > 4096))) return -2;
  const int old = g_chunk_mode;
  g_chunk_mode = mode;
  return old;
}

extern "C" int ulm_memory_chunk_len(int64_t T, int64_t M, int64_t D, int prec) {
  if (T < 0 || M < 0 || D < 0 || (prec != ULM_PREC_BF16 && prec != ULM_PREC_FP32)) return -1;
  return chunk_len(T, M, D, prec);
}

extern "C" int64_t ulm_memory_saved_bytes(int64_t B, int64_t T, int64_t M, int64_t D, int prec) {
  if (B < 0 || T < 0 || M < 0 || D < 0 || (prec != ULM_PREC_BF16 && prec != ULM_PREC_FP32)) return -1;
  const int C = chunk_len(T, M, D, prec);
  const int64_t es = prec == ULM_PREC_FP32 ? 4 : 2;
  if (!C) return B * T * ulm_operand_ld(T) * es;
  return chunk_fwd_layout(nullptr, B, T, M, D, C, prec).bytes;
}

extern "C" int64_t ulm_memory_bwd_work_bytes(int64_t B, int64_t T, int64_t M, int64_t D, int prec) {
  if (B < 0 || T < 0 || M < 0 || D < 0 || (prec != ULM_PREC_BF16 && prec != ULM_PREC_FP32)) return -1;
  const int C = chunk_len(T, M, D, prec);
  const int64_t es = prec == ULM_PREC_FP32 ? 4 : 2;
  if (!C) return B * T * ulm_operand_ld(T) * es;
  return chunk_bwd_layout(nullptr, B, T, M, D, C, prec).bytes;
}

extern "C" int ulm_memory_fwd(const float* r, const float* den, const void* v, int v_dtype, const float* g,
                              const float* w, float* q,
                              void* fast, float* c, void* qop, void* kop, void* vop, void* P, int64_t B, int64_t T,
                              int64_t M, int64_t D, int prec, void* stream) {
  if (int rc = check_prec(prec)) return rc;
  ULM_REQUIRE(B >= 0 && T >= 0 && M >= 0 && D >= 0, "negative extent");
  ULM_REQUIRE(v_dtype == ULM_F32 || v_dtype == ULM_BF16, "v_dtype must be ULM_F32 or ULM_BF16");
  if (B == 0 || T == 0) return ULM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (M == 0) {
    // no slots: q is empty and the fast read is zero
    if (D > 0) {
      ULM_REQUIRE(fast, "null pointer argument");
      ULM_CUDA_TRY(cudaMemsetAsync(fast, 0, B * T * D * elem_size(v_dtype), st));
    }
    return ULM_OK;
  }
  // pointers are checked only where the extents give them elements (an empty tensor's may be null)
  ULM_REQUIRE(r && g && w && q && qop && kop, "null pointer argument");
  const int dt = op_dtype_of(prec);
  const int64_t ldm = ulm_operand_ld(M), ldd = ulm_operand_ld(D), ldt = ulm_operand_ld(T);
  if (int rc = stats_fwd_run(r, den, w, g, q, c, qop, kop, dt, ldm, B, T, M, stream)) return rc;
  if (D == 0) return ULM_OK;
  ULM_REQUIRE(v && fast && vop && P, "null pointer argument");
  if (int rc = convert_rows(v, v_dtype, D, vop, dt, ldd, B * T, D, st)) return rc;
  if (const int C = chunk_len(T, M, D, prec))
    return chunk_read_fwd(qop, kop, vop, g, P, fast, v_dtype, nullptr, nullptr, nullptr, B, T, M, D, C, prec, st);
  if (int rc = ulm_decayed_scores(qop, ldm, kop, ldm, P, ldt, g, B, T, M, prec, stream)) return rc;
  return ulm_causal_apply(P, ldt, vop, ldd, fast, D, v_dtype, 0, B, T, D, prec, stream);
}

// red_st: stream for the statistics backward's dw / dg reductions (nullptr = the caller's stream);
// a caller passing the side stream joins it later (ulm_addressed_memory_bwd)
static int memory_bwd_impl(const float* dq_out, const void* dfast, int do_dtype, const float* r, const float* den,
                           const float* g, const float* w, const float* q, const float* c, const void* qop,
                           const void* kop, const void* vop, const void* P, void* doop, void* dS, float* dqf,
                           float* dk, void* partial, float* dr, void* dv, float* dg, float* dw, int64_t B, int64_t T,
                           int64_t M, int64_t D, int prec, void* stream, cudaStream_t red_st) {
  if (int rc = check_prec(prec)) return rc;
  ULM_REQUIRE(B >= 0 && T >= 0 && M >= 0 && D >= 0, "negative extent");
  ULM_REQUIRE(do_dtype == ULM_F32 || do_dtype == ULM_BF16, "do_dtype must be ULM_F32 or ULM_BF16");
  // pointers are checked only where the extents give them elements (an empty tensor's may be null)
  ULM_REQUIRE(dg && (dw || M == 0), "null pointer argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int dt = op_dtype_of(prec);
  const int64_t ldm = ulm_operand_ld(M), ldd = ulm_operand_ld(D), ldt = ulm_operand_ld(T);
  if (B == 0 || T == 0 || M == 0) {
    if (B * T * D > 0) {
      ULM_REQUIRE(dv, "null pointer argument");
      ULM_CUDA_TRY(cudaMemsetAsync(dv, 0, B * T * D * elem_size(do_dtype), st));
    }
    // nothing reads r or den here
    return ulm_memory_stats_bwd(dqf, dq_out, dk, c ? q : nullptr, c, r, w, g, dr, dw, dg, partial, B, T, M, stream);
  }
  ULM_REQUIRE(dr && r && g && w && qop && kop && dqf && dk && partial, "null pointer argument");
  ULM_REQUIRE(D == 0 || (dfast && dv && vop && P && doop && dS), "null pointer argument");
  if (D == 0) {
    ULM_CUDA_TRY(cudaMemsetAsync(dqf, 0, B * T * M * sizeof(float), st));
    ULM_CUDA_TRY(cudaMemsetAsync(dk, 0, B * T * M * sizeof(float), st));
  } else {
    if (int rc = convert_rows(dfast, do_dtype, D, doop, dt, ldd, B * T, D, st)) return rc;
    if (const int C = chunk_len(T, M, D, prec)) {
      // chunk-carry form: P and dS are the saved and work buffers of that form; the gradient of
      // the q output joins in the statistics backward
      ULM_REQUIRE(B <= 65535 && T < (1ll << 31) && M < (1ll << 31), "extent too large");
      cudaStream_t side = nullptr;
      if (int rc = side_stream(&side)) return rc;
      ChunkBwdLayout CL;
      if (int rc = chunk_read_bwd(doop, qop, kop, vop, g, P, dS, dqf, dk, dv, do_dtype, nullptr, B, T, M, D, C, prec,
                                  st, side, &CL))
        return rc;
      return stats_bwd_run(dqf, dq_out, dk, c ? q : nullptr, c, r, den, w, g, dr, dw, dg, partial, B, T, M, 0,
                           CL.tiles, CL.n_tiles, st, red_st);
    }
    // dS = D * (do v^T): gradient of the scores, same causal decay as the forward; its epilogue
    // also sums (t-s) P dP per tile, the fast read's share of d/dg
    StatsScratch sc = carve_stats_scratch(partial, B, M);
    const int64_t n_tiles = decay_dg_partials(B, T);
    ULM_CUDA_TRY(cudaMemsetAsync(sc.tiles, 0, n_tiles * sizeof(float), st));
    // dv = P^T do and dk = dS^T q run on the side stream beside dS and dq; dS and dq are launched
    // first, so the chain dS -> dq -> statistics gets the SMs first
    cudaStream_t side = nullptr;
    if (int rc = side_stream(&side)) return rc;
    if (int rc = stream_after(side, st)) return rc;
    {
      Operand A{doop, ldd, T * ldd, D, T, dt, false};
      Operand Bo{vop, ldd, T * ldd, D, T, dt, false};
      GemmShape s{(int)B, (int)T, (int)T, (int)D, CAUSAL_NLOWER};
      GemmEpilogue e = make_epilogue(EPI_DECAY_DG, dt, dS, ldt, T * ldt, g);
      e.aux = P;
      e.ld_aux = ldt;
      e.aux_bstride = T * ldt;
      e.tile_partial = sc.tiles;
      e.vec_ok = e.vec_ok && is_aligned16(P);
      if (int rc = run_gemm(A, Bo, s, e, st)) return rc;
    }
    if (int rc = ulm_causal_apply(P, ldt, doop, ldd, dv, D, do_dtype, 1, B, T, D, prec, side)) return rc;
    if (int rc = stream_after(side, st)) return rc;  // dS is ready for dk
    {
      // dq = dS k, with the gradient of the q output added in the epilogue: the statistics backward
      // only needs the sum (fast_identity = 0 below)
      Operand A{dS, ldt, T * ldt, T, T, dt, false};
      Operand Bo{kop, ldm, T * ldm, M, T, dt, true};
      GemmShape s{(int)B, (int)T, (int)M, (int)T, CAUSAL_KLOWER};
      GemmEpilogue e = make_epilogue(dq_out ? EPI_STORE_ADD : EPI_STORE, ULM_F32, dqf, M, T * M, nullptr);
      if (dq_out) {
        e.aux = dq_out;
        e.ld_aux = M;
        e.aux_bstride = T * M;
        e.vec_ok = e.vec_ok && is_aligned16(dq_out);
      }
      if (int rc = run_gemm(A, Bo, s, e, st)) return rc;
    }
    if (int rc = ulm_causal_apply(dS, ldt, qop, ldm, dk, M, ULM_F32, 1, B, T, M, prec, side)) return rc;
    if (int rc = stream_after(st, side)) return rc;  // join: dk and dv are done
    ULM_REQUIRE(B <= 65535 && T < (1ll << 31) && M < (1ll << 31), "extent too large");
    // without a saved c the statistics backward rebuilds q and c from r (TMA scan path)
    return stats_bwd_run(dqf, nullptr, dk, c ? q : nullptr, c, r, den, w, g, dr, dw, dg, partial, B, T, M, 0,
                         sc.tiles, n_tiles, st, red_st);
  }
  return stats_bwd_run(dqf, dq_out, dk, c ? q : nullptr, c, r, den, w, g, dr, dw, dg, partial, B, T, M, 1, nullptr, 0,
                       st, red_st);
}

extern "C" int ulm_memory_bwd(const float* dq_out, const void* dfast, int do_dtype, const float* r, const float* den,
                              const float* g, const float* w, const float* q, const float* c, const void* qop, const void* kop,
                              const void* vop, const void* P, void* doop, void* dS, float* dqf, float* dk,
                              void* partial, float* dr, void* dv, float* dg, float* dw, int64_t B, int64_t T,
                              int64_t M, int64_t D, int prec, void* stream) {
  return memory_bwd_impl(dq_out, dfast, do_dtype, r, den, g, w, q, c, qop, kop, vop, P, doop, dS, dqf, dk, partial, dr,
                         dv, dg, dw, B, T, M, D, prec, stream, nullptr);
}

// ---- the block's combine fused into the fast memory (model.py:79-85) -------------------------------
namespace ulm {
namespace {

// Split of a contraction over `rows` into S k ranges so an (N1 x N2) product fills the CTA pairs once
// (S x tiles <= pairs), at most 8, each range at least 1024 rows and none empty.
int fill_split(int64_t rows, int64_t N1, int64_t N2) {
  const int dev = current_device();
  const int pairs = (dev >= 0 ? sm_count(dev) : 148) / 2;
  const int64_t tiles = cdiv(N1, 256) * cdiv(N2, 256);
  int S = (int)std::max<int64_t>(1, std::min<int64_t>(8, pairs / std::max<int64_t>(1, tiles)));
  while (S > 1 && (rows / S < 1024 || (int64_t)(S - 1) * ksplit_chunk((int)rows, S) >= rows)) --S;
  return S;
}

}  // namespace
}  // namespace ulm

extern "C" int64_t ulm_combine_grad_scratch(int64_t B, int64_t T, int64_t M, int64_t D) {
  if (B < 0 || T < 0 || M < 0 || D < 0) return -1;
  // split-K partials of G, sized for the largest split, then the dw partials per row block
  return (8 * D * M + cdiv(D, COMBINE_ROWS) * M) * (int64_t)sizeof(float);
}

extern "C" int ulm_memory_combine_fwd(const float* r, const float* den, const void* v, int v_dtype, const float* g,
                                      const float* w, const float* mu, const void* x, int x_dtype, void* y, float* q,
                                      float* c, void* qop, void* kop, void* vop, void* P, void* wmu, int64_t B,
                                      int64_t T, int64_t M, int64_t D, int prec, void* stream) {
  if (int rc = check_prec(prec)) return rc;
  ULM_REQUIRE(B >= 0 && T >= 0 && M >= 0 && D >= 0, "negative extent");
  ULM_REQUIRE(v_dtype == ULM_F32 || v_dtype == ULM_BF16, "v_dtype must be ULM_F32 or ULM_BF16");
  ULM_REQUIRE(x_dtype == ULM_F32 || x_dtype == ULM_BF16, "x_dtype must be ULM_F32 or ULM_BF16");
  if (B == 0 || T == 0 || D == 0) return ULM_OK;
  ULM_REQUIRE(v && x && y && g && w, "null pointer argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (M == 0) return convert_rows(x, x_dtype, D, y, x_dtype, D, B * T, D, st);  // no slots: y = x
  ULM_REQUIRE(r && mu && qop && kop && vop && P && wmu, "null pointer argument");
  ULM_REQUIRE(B <= 65535 && T < (1 << 30) && M < (1 << 30) && D < (1 << 30), "extent too large");
  const int dt = op_dtype_of(prec);
  const int64_t ldm = ulm_operand_ld(M), ldd = ulm_operand_ld(D), ldt = ulm_operand_ld(T);
  if (int rc = stats_fwd_run(r, den, w, g, q, c, qop, kop, dt, ldm, B, T, M, stream)) return rc;
  if (int rc = convert_rows(v, v_dtype, D, vop, dt, ldd, B * T, D, st)) return rc;
  combine_weight_t_kernel<<<dim3((unsigned)cdiv(M, 32), (unsigned)cdiv(D, 32)), 256, 0, st>>>(mu, w, wmu, dt, ldd,
                                                                                            (int)D, (int)M);
  ULM_LAUNCH_CHECK("combine_weight_t_kernel");
  if (const int C = chunk_len(T, M, D, prec))
    return chunk_read_fwd(qop, kop, vop, g, P, y, x_dtype, x, wmu, nullptr, B, T, M, D, C, prec, st);
  if (int rc = ulm_decayed_scores(qop, ldm, kop, ldm, P, ldt, g, B, T, M, prec, stream)) return rc;
  // y = x + P v (causal k range) + q (w mu)^T (all M) in one accumulator
  Operand A{P, ldt, T * ldt, T, T, dt, false};
  Operand Bv{vop, ldd, T * ldd, D, T, dt, true};
  Operand A2{qop, ldm, T * ldm, M, T, dt, false};
  Operand B2{wmu, ldd, 0, D, M, dt, true};
  GemmShape s{(int)B, (int)T, (int)D, (int)T, CAUSAL_KLOWER};
  s.K2 = (int)M;
  GemmEpilogue e = make_epilogue(EPI_STORE_ADD, x_dtype, y, D, T * D, nullptr);
  e.aux = x;
  e.ld_aux = D;
  e.aux_bstride = T * D;
  e.vec_ok = e.vec_ok && is_aligned16(x);
  return run_gemm2(A, Bv, &A2, &B2, s, e, st);
}

static int combine_bwd_impl(const void* dy, int dy_dtype, const float* r, const float* den, const float* g,
                            const float* w, const float* mu, const float* q, const float* c, const void* qop,
                            const void* kop, const void* vop, const void* P, void* doop, void* dS, void* mw, float* dqf,
                            float* dk, void* partial, float* gpart, float* dr, void* dv, int dv_dtype, float* dg,
                            float* dw, float* dmu, int64_t B, int64_t T, int64_t M, int64_t D, int prec, void* stream,
                            cudaStream_t red_st) {
  if (int rc = check_prec(prec)) return rc;
  ULM_REQUIRE(B >= 0 && T >= 0 && M >= 0 && D >= 0, "negative extent");
  ULM_REQUIRE(dy_dtype == ULM_F32 || dy_dtype == ULM_BF16, "dy_dtype must be ULM_F32 or ULM_BF16");
  ULM_REQUIRE(dv_dtype == ULM_F32 || dv_dtype == ULM_BF16, "dv_dtype must be ULM_F32 or ULM_BF16");
  ULM_REQUIRE(dy && dr && dv && dg && dw && dmu, "null pointer argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B == 0 || T == 0 || M == 0 || D == 0) {
    if (B * T * D > 0) ULM_CUDA_TRY(cudaMemsetAsync(dv, 0, B * T * D * elem_size(dv_dtype), st));
    if (D * M > 0) ULM_CUDA_TRY(cudaMemsetAsync(dmu, 0, D * M * sizeof(float), st));
    return ulm_memory_stats_bwd(dqf, nullptr, dk, c ? q : nullptr, c, r, w, g, dr, dw, dg, partial, B, T, M, stream);
  }
  ULM_REQUIRE(r && g && w && mu && qop && kop && vop && P && doop && dS && mw && dqf && dk && partial && gpart,
              "null pointer argument");
  ULM_REQUIRE(B <= 65535 && T < (1 << 30) && M < (1 << 30) && D < (1 << 30), "extent too large");
  const int dt = op_dtype_of(prec);
  const int64_t ldm = ulm_operand_ld(M), ldd = ulm_operand_ld(D), ldt = ulm_operand_ld(T);
  // dfast = dy: its operand copy is the A operand of the score gradient, of dv and of d(q w)
  if (int rc = convert_rows(dy, dy_dtype, D, doop, dt, ldd, B * T, D, st)) return rc;
  float* dw_part = gpart + 8 * D * M;
  const unsigned row_blocks = (unsigned)cdiv(D, COMBINE_ROWS);
  // G = dy^T q over all B*T rows (split K), then dmu = G w and the combine's share of dw,
  // sum_d mu G (partials, added to dw after the statistics backward)
  auto combine_grads = [&](cudaStream_t on) -> int {
    const int64_t rows = B * T;
    const int S = fill_split(rows, D, M);
    Operand A{doop, ldd, 0, D, rows, dt, true};
    Operand Bq{qop, ldm, 0, M, rows, dt, true};
    GemmShape s{S, (int)D, (int)M, (int)rows, CAUSAL_NONE};
    s.ksplit = S;
    GemmEpilogue e = make_epilogue(EPI_STORE, ULM_F32, gpart, M, D * M, nullptr);
    if (int rc = run_gemm(A, Bq, s, e, on)) return rc;
    combine_grad_kernel<<<dim3((unsigned)cdiv(M, 32), row_blocks), 256, 0, on>>>(gpart, S, mu, w, dmu, dw_part,
                                                                                (int)D, (int)M);
    ULM_LAUNCH_CHECK("combine_grad_kernel");
    return ULM_OK;
  };
  if (const int C = chunk_len(T, M, D, prec)) {
    // chunk-carry form (P and dS are its saved and work buffers)
    cudaStream_t side = nullptr;
    if (int rc = side_stream(&side)) return rc;
    combine_weight_kernel<<<(unsigned)std::min<int64_t>(cdiv(D * M, 256), 8 * 148), 256, 0, st>>>(mu, w, mw, dt, ldm,
                                                                                               (int)D, (int)M);
    ULM_LAUNCH_CHECK("combine_weight_kernel");
    if (int rc = stream_after(side, st)) return rc;
    if (int rc = combine_grads(side)) return rc;
    ChunkBwdLayout CL;
    if (int rc = chunk_read_bwd(doop, qop, kop, vop, g, P, dS, dqf, dk, dv, dv_dtype, mw, B, T, M, D, C, prec, st,
                                side, &CL))
      return rc;  // joins the side stream
    if (int rc = stats_bwd_run(dqf, nullptr, dk, c ? q : nullptr, c, r, den, w, g, dr, dw, dg, partial, B, T, M, 0,
                               CL.tiles, CL.n_tiles, st, red_st))
      return rc;
    add_parts_kernel<<<(unsigned)cdiv(M, 256), 256, 0, red_st ? red_st : st>>>(dw_part, (int)row_blocks, M, dw);
    ULM_LAUNCH_CHECK("add_parts_kernel");
    return ULM_OK;
  }
  StatsScratch sc = carve_stats_scratch(partial, B, M);
  const int64_t n_tiles = decay_dg_partials(B, T);
  ULM_CUDA_TRY(cudaMemsetAsync(sc.tiles, 0, n_tiles * sizeof(float), st));
  // side stream: dv and G = dy^T q beside dS and dq, then dk
  cudaStream_t side = nullptr;
  if (int rc = side_stream(&side)) return rc;
  if (int rc = stream_after(side, st)) return rc;
  {
    Operand A{doop, ldd, T * ldd, D, T, dt, false};
    Operand Bo{vop, ldd, T * ldd, D, T, dt, false};
    GemmShape s{(int)B, (int)T, (int)T, (int)D, CAUSAL_NLOWER};
    GemmEpilogue e = make_epilogue(EPI_DECAY_DG, dt, dS, ldt, T * ldt, g);
    e.aux = P;
    e.ld_aux = ldt;
    e.aux_bstride = T * ldt;
    e.tile_partial = sc.tiles;
    e.vec_ok = e.vec_ok && is_aligned16(P);
    if (int rc = run_gemm(A, Bo, s, e, st)) return rc;
  }
  if (int rc = ulm_causal_apply(P, ldt, doop, ldd, dv, D, dv_dtype, 1, B, T, D, prec, side)) return rc;
  if (int rc = combine_grads(side)) return rc;
  if (int rc = stream_after(side, st)) return rc;  // dS is ready for dk
  combine_weight_kernel<<<(unsigned)std::min<int64_t>(cdiv(D * M, 256), 8 * 148), 256, 0, st>>>(mu, w, mw, dt, ldm,
                                                                                             (int)D, (int)M);
  ULM_LAUNCH_CHECK("combine_weight_kernel");
  {
    // dq = dS k + dy (mu w): the gradient reaching q through the combine joins the product
    Operand A{dS, ldt, T * ldt, T, T, dt, false};
    Operand Bk{kop, ldm, T * ldm, M, T, dt, true};
    Operand A2{doop, ldd, T * ldd, D, T, dt, false};
    Operand B2{mw, ldm, 0, M, D, dt, true};
    GemmShape s{(int)B, (int)T, (int)M, (int)T, CAUSAL_KLOWER};
    s.K2 = (int)D;
    GemmEpilogue e = make_epilogue(EPI_STORE, ULM_F32, dqf, M, T * M, nullptr);
    if (int rc = run_gemm2(A, Bk, &A2, &B2, s, e, st)) return rc;
  }
  if (int rc = ulm_causal_apply(dS, ldt, qop, ldm, dk, M, ULM_F32, 1, B, T, M, prec, side)) return rc;
  if (int rc = stream_after(st, side)) return rc;  // dk, dv and the combine's partials are done
  if (int rc = stats_bwd_run(dqf, nullptr, dk, c ? q : nullptr, c, r, den, w, g, dr, dw, dg, partial, B, T, M, 0,
                             sc.tiles, n_tiles, st, red_st))
    return rc;
  {
    // on the stream of the dw reduction it adds to
    add_parts_kernel<<<(unsigned)cdiv(M, 256), 256, 0, red_st ? red_st : st>>>(dw_part, (int)row_blocks, M, dw);
    ULM_LAUNCH_CHECK("add_parts_kernel");
  }
  return ULM_OK;
}

extern "C" int ulm_memory_combine_bwd(const void* dy, int dy_dtype, const float* r, const float* den, const float* g,
                                      const float* w, const float* mu, const float* q, const float* c,
                                      const void* qop, const void* kop, const void* vop, const void* P, void* doop,
                                      void* dS, void* mw, float* dqf, float* dk, void* partial, float* gpart,
                                      float* dr, void* dv, int dv_dtype, float* dg, float* dw, float* dmu,
                                      int64_t B, int64_t T, int64_t M, int64_t D, int prec, void* stream) {
  return combine_bwd_impl(dy, dy_dtype, r, den, g, w, mu, q, c, qop, kop, vop, P, doop, dS, mw, dqf, dk, partial,
                          gpart, dr, dv, dv_dtype, dg, dw, dmu, B, T, M, D, prec, stream, nullptr);
}
