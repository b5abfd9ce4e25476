// Batched recurrent decode: UnifiedBlock.step (model.py:96-111) / run.c forward (run.c:193-265) for
// B sequences at once, one token per call.
//
// Per block and token, for every sequence b (lam, eps scalars; w, mu per slot):
//   h = RMSNorm(x)                          decode_prologue_kernel
//   u = conv(window(buf), h), buf <- shift  decode_prologue_kernel
//   a = K u + bias, v = W_v h               batched GEMMs (gemm.cu: fp32 FMA or tcgen05 bf16)
//   z = relu(a)^2, r = z / (eps + sum z)    decode_address_kernel
//   c = lam c + (1-lam) w + r_prev, q = r/c decode_address_kernel
//   r_prev <- r (the old r_prev to work)    decode_address_kernel
//   U = lam U + (1-lam) mu w + v r_old^T    decode_state_kernel (U read once, written once)
//   x += U q                                decode_state_kernel
// The state U (B x D x M fp32 per block) is the only large traffic: 8 D M bytes per sequence per
// block per token; every other tensor is O(B (D + M)) or a weight shared by the whole batch.
//
// fp32 mode keeps run.c's operation order for the state update, ((lam U) + (1-lam) mu w) + v r_prev,
// with the constant middle term precomputed once per block by ulm_decode_prepare_block, and no
// fused multiply-adds, so the state evolves as in run.c up to the order of the dot-product sums.
#include <algorithm>
#include <cstring>

#include "gemm.cuh"

namespace ulm {

constexpr int DEC_THREADS = 256;
// The per-row kernels (prologue, address, final norm, greedy pick) run one CTA per sequence: 1024
// threads at small batches, where a few CTAs hold the GPU and each must cover its row in one round
// of loads, 256 from 64 sequences on.
constexpr int DEC_ROW_MAX_THREADS = 1024;
inline int dec_row_threads(int64_t B) { return B < 64 ? DEC_ROW_MAX_THREADS : DEC_THREADS; }

__device__ __forceinline__ float block_sum(float v, float* red) {
  // sum over the block, fixed order
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  if (lane == 0) red[wp] = v;
  __syncthreads();
  float s = 0.f;
  if (threadIdx.x == 0) {
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += red[i];
    red[32] = s;
  }
  __syncthreads();
  s = red[32];
  __syncthreads();
  return s;
}

// h = rmsnorm(x) * norm_w; u = conv over the window (buf oldest..newest, h); buf shifts.
// Also writes bf16 copies of h and u when hop/uop are given (tensor-core GEMM operands).
__global__ void __launch_bounds__(DEC_ROW_MAX_THREADS)
    decode_prologue_kernel(const float* __restrict__ x, const float* __restrict__ norm_w,
                           const float* __restrict__ conv_w, float* __restrict__ buf, float* __restrict__ h,
                           float* __restrict__ u, __nv_bfloat16* __restrict__ hop, __nv_bfloat16* __restrict__ uop,
                           int64_t ld_op, int D, int K, float norm_eps) {
  pdl_enter();
  __shared__ float red[33];
  const int b = blockIdx.x;
  const float* xb = x + (int64_t)b * D;
  float ss = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) ss = __fadd_rn(ss, __fmul_rn(xb[i], xb[i]));
  ss = block_sum(ss, red);
  const float scale = 1.0f / sqrtf(ss / (float)D + norm_eps);
  const int kw = K - 1;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const float hv = norm_w[i] * (scale * xb[i]);
    h[(int64_t)b * D + i] = hv;
    float* st = buf + ((int64_t)b * D + i) * kw;
    const float* cw = conv_w + (int64_t)i * K;
    float uv = __fmul_rn(cw[kw], hv);
    for (int j = 0; j < kw; ++j) uv = __fadd_rn(uv, __fmul_rn(cw[j], st[j]));
    for (int j = 0; j + 1 < kw; ++j) st[j] = st[j + 1];
    if (kw > 0) st[kw - 1] = hv;
    u[(int64_t)b * D + i] = uv;
    if (hop) hop[(int64_t)b * ld_op + i] = __float2bfloat16_rn(hv);
    if (uop) uop[(int64_t)b * ld_op + i] = __float2bfloat16_rn(uv);
  }
}

// r = relu(a + bias)^2 / (eps + sum), c = lam c + (1-lam) w + r_prev, q = r / c; then r_prev <- r,
// the old r_prev going to r_old for the state update (each slot is read and written by one thread,
// so the state needs no separate copy of r after its update)
__global__ void __launch_bounds__(DEC_ROW_MAX_THREADS)
    decode_address_kernel(const float* __restrict__ a, const float* __restrict__ key_b, const float* __restrict__ w,
                          const float* __restrict__ lam_p, const float* __restrict__ eps_p, float* __restrict__ c,
                          float* __restrict__ r_prev, float* __restrict__ r_old, float* __restrict__ q, int M) {
  pdl_enter();
  __shared__ float red[33];
  const int b = blockIdx.x;
  const float lam = *lam_p, eps = *eps_p;
  const int64_t o = (int64_t)b * M;
  float zs = 0.f;
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    float z = a[o + m] + key_b[m];
    z = z > 0.f ? z * z : 0.f;
    r_old[o + m] = z;  // z until the second loop
    zs += z;
  }
  zs = block_sum(zs, red);
  const float denom = eps + zs;
  const float one_minus = 1.0f - lam;
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    const float r = r_old[o + m] / denom;
    const float rp = r_prev[o + m];
    const float cc = __fadd_rn(__fadd_rn(__fmul_rn(lam, c[o + m]), __fmul_rn(one_minus, w[m])), rp);
    c[o + m] = cc;
    q[o + m] = r / cc;
    r_old[o + m] = rp;
    r_prev[o + m] = r;
  }
}

// S warps per state row (b, d) (S in {1, 2, 4, 8}; more at small batches, so that enough loads are in
// flight): U'[m] = ((lam U) + prior[d][m]) + v[d] r_prev[m]; x[b][d] += sum U' q. prior = (1-lam) mu w,
// fp32 or bf16. The row is streamed once with 16-byte loads and stores; a CTA's 8 warps cover 8 / S
// rows and the S partial dot products of a row are added in warp order through shared memory.
template <typename PriorT, int S>
__global__ void __launch_bounds__(DEC_THREADS)
    decode_state_kernel(float* __restrict__ U, const PriorT* __restrict__ prior, const float* __restrict__ v,
                        const float* __restrict__ r_prev, const float* __restrict__ q, const float* __restrict__ lam_p,
                        float* __restrict__ x, int D, int M) {
  pdl_enter();
  __shared__ float red[DEC_THREADS / 32];
  constexpr int warps = DEC_THREADS / 32;
  const int wp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = wp % S;
  const int64_t row = (int64_t)blockIdx.x * (warps / S) + wp / S;  // b * D + d
  const int b = (int)(row / D);
  const int d = (int)(row - (int64_t)b * D);
  const float lam = *lam_p;
  const float vd = v[row];
  float* Ur = U + row * M;
  const PriorT* pr = prior + (int64_t)d * M;
  const float* rp = r_prev + (int64_t)b * M;
  const float* qb = q + (int64_t)b * M;
  float acc = 0.f;
  for (int m = (sub * 32 + lane) * 4; m < M; m += 128 * S) {
    float4 u4 = *reinterpret_cast<const float4*>(Ur + m);
    const float4 r4 = *reinterpret_cast<const float4*>(rp + m);
    const float4 q4 = *reinterpret_cast<const float4*>(qb + m);
    float p0, p1, p2, p3;
    if constexpr (sizeof(PriorT) == 4) {
      const float4 p4 = *reinterpret_cast<const float4*>(pr + m);
      p0 = p4.x; p1 = p4.y; p2 = p4.z; p3 = p4.w;
    } else {
      const uint2 raw = *reinterpret_cast<const uint2*>(pr + m);
      __nv_bfloat162 h0, h1;
      memcpy(&h0, &raw.x, 4);
      memcpy(&h1, &raw.y, 4);
      const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
      p0 = f0.x; p1 = f0.y; p2 = f1.x; p3 = f1.y;
    }
    u4.x = __fadd_rn(__fadd_rn(__fmul_rn(lam, u4.x), p0), __fmul_rn(vd, r4.x));
    u4.y = __fadd_rn(__fadd_rn(__fmul_rn(lam, u4.y), p1), __fmul_rn(vd, r4.y));
    u4.z = __fadd_rn(__fadd_rn(__fmul_rn(lam, u4.z), p2), __fmul_rn(vd, r4.z));
    u4.w = __fadd_rn(__fadd_rn(__fmul_rn(lam, u4.w), p3), __fmul_rn(vd, r4.w));
    *reinterpret_cast<float4*>(Ur + m) = u4;
    acc = fmaf(u4.x, q4.x, acc);
    acc = fmaf(u4.y, q4.y, acc);
    acc = fmaf(u4.z, q4.z, acc);
    acc = fmaf(u4.w, q4.w, acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if constexpr (S == 1) {
    if (lane == 0) x[row] += acc;
    return;
  }
  if (lane == 0) red[wp] = acc;
  __syncthreads();
  if (sub == 0 && lane == 0) {
    float t = red[wp];
    for (int j = 1; j < S; ++j) t += red[wp + j];
    x[row] += t;
  }
}

// prior[d][m] = ((1 - lam) * mu[d][m]) * w[m], and the initial state U = mu * w (run.c:121-138)
__global__ void decode_prepare_kernel(const float* __restrict__ mu, const float* __restrict__ w,
                                      const float* __restrict__ lam_p, void* __restrict__ prior, int prior_bf16,
                                      int D, int M) {
  const float lam = *lam_p;
  const int64_t n = (int64_t)D * M;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int m = (int)(i % M);
    const float p = __fmul_rn(__fmul_rn(1.0f - lam, mu[i]), w[m]);
    if (prior_bf16)
      static_cast<__nv_bfloat16*>(prior)[i] = __float2bfloat16_rn(p);
    else
      static_cast<float*>(prior)[i] = p;
  }
}

__global__ void decode_reset_kernel(const float* __restrict__ mu, const float* __restrict__ w, float* __restrict__ U,
                                    float* __restrict__ c, float* __restrict__ r_prev, float* __restrict__ buf,
                                    int B, int D, int M, int kw) {
  const int64_t nU = (int64_t)B * D * M;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nU; i += stride) {
    const int64_t dm = i % ((int64_t)D * M);
    U[i] = mu[dm] * w[dm % M];
  }
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)B * M; i += stride) {
    c[i] = w[i % M];
    r_prev[i] = 0.f;
  }
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)B * D * kw; i += stride) buf[i] = 0.f;
}

// final RMSNorm of the residual stream, fp32 and optional bf16 copy
__global__ void __launch_bounds__(DEC_ROW_MAX_THREADS)
    decode_final_norm_kernel(const float* __restrict__ x, const float* __restrict__ norm_w, float* __restrict__ xn,
                             __nv_bfloat16* __restrict__ xop, int64_t ld_op, int D, float norm_eps) {
  pdl_enter();
  __shared__ float red[33];
  const int b = blockIdx.x;
  const float* xb = x + (int64_t)b * D;
  float ss = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) ss += xb[i] * xb[i];
  ss = block_sum(ss, red);
  const float scale = 1.0f / sqrtf(ss / (float)D + norm_eps);
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const float v = norm_w[i] * (scale * xb[i]);
    xn[(int64_t)b * D + i] = v;
    if (xop) xop[(int64_t)b * ld_op + i] = __float2bfloat16_rn(v);
  }
}

// greedy pick: first index of the largest logit (run.c sample_argmax), then gather the next
// token's embedding row into x. Each thread keeps the first index of its largest value (16-byte
// loads when the rows allow them), then a tree keeps the larger value, the smaller index on ties.
__device__ __forceinline__ void argmax_take(float v, int i, float& best, int& idx) {
  if (v > best || (v == best && i < idx)) {
    best = v;
    idx = i;
  }
}

__global__ void __launch_bounds__(DEC_ROW_MAX_THREADS)
    decode_argmax_embed_kernel(const float* __restrict__ logits, int64_t ld_logits, int V,
                               const void* __restrict__ emb, int emb_bf16, int D, int* __restrict__ next_token,
                               float* __restrict__ x) {
  pdl_enter();
  __shared__ float bv[DEC_ROW_MAX_THREADS];
  __shared__ int bi[DEC_ROW_MAX_THREADS];
  const int b = blockIdx.x;
  const float* lg = logits + (int64_t)b * ld_logits;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  if ((reinterpret_cast<uintptr_t>(lg) & 15u) == 0) {
    const int V4 = V / 4;
    const float4* l4 = reinterpret_cast<const float4*>(lg);
#pragma unroll 4
    for (int j = threadIdx.x; j < V4; j += blockDim.x) {
      const float4 v = l4[j];
      argmax_take(v.x, 4 * j, best, idx);
      argmax_take(v.y, 4 * j + 1, best, idx);
      argmax_take(v.z, 4 * j + 2, best, idx);
      argmax_take(v.w, 4 * j + 3, best, idx);
    }
    for (int i = 4 * V4 + threadIdx.x; i < V; i += blockDim.x) argmax_take(lg[i], i, best, idx);
  } else {
    for (int i = threadIdx.x; i < V; i += blockDim.x) argmax_take(lg[i], i, best, idx);
  }
  bv[threadIdx.x] = best;
  bi[threadIdx.x] = idx;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if ((int)threadIdx.x < s) {
      const float ov = bv[threadIdx.x + s];
      const int oi = bi[threadIdx.x + s];
      if (ov > bv[threadIdx.x] || (ov == bv[threadIdx.x] && oi < bi[threadIdx.x])) {
        bv[threadIdx.x] = ov;
        bi[threadIdx.x] = oi;
      }
    }
    __syncthreads();
  }
  const int tok = bi[0] == 0x7fffffff ? 0 : bi[0];
  if (threadIdx.x == 0) next_token[b] = tok;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const int64_t o = (int64_t)tok * D + i;
    x[(int64_t)b * D + i] = emb_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(emb)[o])
                                     : static_cast<const float*>(emb)[o];
  }
}

__global__ void decode_embed_kernel(const int* __restrict__ tokens, const void* __restrict__ emb, int emb_bf16, int D,
                                    float* __restrict__ x) {
  pdl_enter();
  const int b = blockIdx.x;
  const int tok = tokens[b];
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const int64_t o = (int64_t)tok * D + i;
    x[(int64_t)b * D + i] = emb_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(emb)[o])
                                     : static_cast<const float*>(emb)[o];
  }
}

// ---- parallel prefill: the decode state after a whole prompt ----------------------------------
// After the training-form forward of a block over T prompt positions (z, den from ulm_address_fwd
// with normalize = 0; kop, vop the operand copies of ulm_memory_fwd / ulm_memory_combine_fwd), the
// block's recurrent state is what UnifiedBlock.step (model.py:96-111) leaves after those T tokens:
//   U = w mu + sum_s lam^(T-1-s) v_s k_s^T   (k_s = r_{s-1}),   c = w + sum_s lam^(T-1-s) k_s,
//   r_prev = r_{T-1},   buf = the last K-1 normalised inputs h, oldest first.
// The sum over s is one carry product with a single chunk of T positions (the values scaled by
// lam^(T-1-s), the state rows the value channels so it lands in the decoder's (D, M) layout).

// c (run's update order c = (lam c + (1-lam) w) + r_prev from c = w) and r_prev; one thread per slot
__global__ void decode_prefill_stats_kernel(const float* __restrict__ z, const float* __restrict__ den,
                                            const float* __restrict__ w, const float* __restrict__ lam_p,
                                            float* __restrict__ c, float* __restrict__ r_prev, int T, int M) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (m >= M) return;
  const float lam = *lam_p, one_minus = 1.0f - lam, wm = w[m];
  const float* zb = z + (int64_t)b * T * M;
  const float* db = den + (int64_t)b * T;
  float cc = wm, rp = 0.f;
  for (int t = 0; t < T; ++t) {
    cc = __fadd_rn(__fadd_rn(__fmul_rn(lam, cc), __fmul_rn(one_minus, wm)), rp);
    rp = zb[(int64_t)t * M + m] / db[t];
  }
  c[(int64_t)b * M + m] = cc;
  r_prev[(int64_t)b * M + m] = rp;
}

// U[b] += w mu (the prior part of the state); buf[b][d][j] = h[b][T-kw+j][d] (0 before position 0)
__global__ void decode_prefill_state_kernel(float* __restrict__ U, const float* __restrict__ mu,
                                            const float* __restrict__ w, const void* __restrict__ h, int h_bf16,
                                            float* __restrict__ buf, int B, int T, int D, int M, int kw) {
  const int64_t nU = (int64_t)B * D * M;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nU; i += stride) {
    const int64_t dm = i % ((int64_t)D * M);
    U[i] = mu[dm] * w[dm % M] + U[i];
  }
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)B * D * kw; i += stride) {
    const int64_t b = i / ((int64_t)D * kw), rem = i - b * D * kw;
    const int d = (int)(rem / kw), j = (int)(rem - (int64_t)d * kw);
    const int t = T - kw + j;
    float val = 0.f;
    if (t >= 0) {
      const int64_t off = ((int64_t)b * T + t) * D + d;
      val = h_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(h)[off]) : static_cast<const float*>(h)[off];
    }
    buf[i] = val;
  }
}

}  // namespace ulm

extern "C" int64_t ulm_decode_prefill_work_bytes(int64_t B, int64_t T, int64_t D, int prec) {
  if (B < 0 || T < 0 || D < 0 || (prec != ULM_PREC_BF16 && prec != ULM_PREC_FP32)) return -1;
  return B * T * ulm_operand_ld(D) * (prec == ULM_PREC_FP32 ? 4 : 2);
}

extern "C" int ulm_decode_prefill_block(const void* kop, const void* vop, const float* g, const float* lam,
                                        const float* z, const float* den, const void* h, int h_dtype,
                                        const float* mu, const float* w, void* work, float* U, float* c,
                                        float* r_prev, float* buf, int64_t B, int64_t T, int64_t D, int64_t M,
                                        int64_t conv_size, int prec, void* stream) {
  ULM_REQUIRE(prec == ULM_PREC_BF16 || prec == ULM_PREC_FP32, "prec must be ULM_PREC_BF16 or ULM_PREC_FP32");
  ULM_REQUIRE(h_dtype == ULM_F32 || h_dtype == ULM_BF16, "h_dtype must be ULM_F32 or ULM_BF16");
  ULM_REQUIRE(B > 0 && T > 0 && D > 0 && M > 0 && conv_size >= 1, "bad extents");
  ULM_REQUIRE(B <= 65535 && T < (1 << 30) && D < (1 << 30) && M < (1 << 30), "extent too large");
  ULM_REQUIRE(kop && vop && g && lam && z && den && h && mu && w && work && U && c && r_prev &&
                  (buf || conv_size <= 1),
              "null pointer argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int dt = op_dtype_of(prec);
  const int64_t ldm = ulm_operand_ld(M), ldd = ulm_operand_ld(D);
  // the values scaled by lam^(T-1-s): one chunk of T positions
  if (int rc = chunk_scale_rows(vop, work, dt, ldd, B * T, D, (int)T, g, (float)(T - 1), -1.f, st)) return rc;
  {
    // U[b][d][m] = sum_s vhat_s[d] k_s[m]: state rows d (A = vhat as [pos][d]), columns m (B = k)
    Operand A{work, ldd, T * ldd, D, T, dt, true};
    Operand Bk{kop, ldm, T * ldm, M, T, dt, true};
    GemmShape s{(int)B, (int)D, (int)M, (int)T, CAUSAL_NONE};
    s.carry = CARRY_FWD;
    s.carry_C = (int)T;
    s.carry_chunks = 1;
    s.carry_end = 1;
    GemmEpilogue e = make_epilogue(EPI_STORE, ULM_F32, U, M, D * M, g);
    e.end_state = U;
    e.end_ld = M;
    e.end_bstride = D * M;
    if (int rc = run_gemm(A, Bk, s, e, st)) return rc;
  }
  decode_prefill_stats_kernel<<<dim3((unsigned)cdiv(M, 256), (unsigned)B), 256, 0, st>>>(z, den, w, lam, c, r_prev,
                                                                                       (int)T, (int)M);
  ULM_LAUNCH_CHECK("decode_prefill_stats_kernel");
  decode_prefill_state_kernel<<<(unsigned)std::min<int64_t>(cdiv(B * D * M, 256), 8 * 148), 256, 0, st>>>(
      U, mu, w, h, h_dtype == ULM_BF16, buf, (int)B, (int)T, (int)D, (int)M, (int)(conv_size - 1));
  ULM_LAUNCH_CHECK("decode_prefill_state_kernel");
  return ULM_OK;
}



using namespace ulm;

namespace {

int weight_dtype_ok(int dt) { return dt == ULM_F32 || dt == ULM_BF16; }

}  // namespace

namespace ulm {

// Small-batch decode GEMM with bf16 weights: out[b][n] = sum_k x[b][k] W[n][k] for B <= GEMV_MAX_B.
// The weights are streamed once by every warp of a grid that covers all SMs (one warp per weight
// row at a time, 16-byte loads, fp32 accumulators), the batch's rows of x sit in shared memory in
// fp32; a tensor-core tile of 128 rows would leave most of its rows empty and spread the weight
// reads over only N / 128 CTAs.
constexpr int GEMV_MAX_B = 4;
constexpr int GEMV_WARPS = 8;

// Up to two products per launch (the key and val projections of a decode step share one): rows
// [0, N1) of the grid's row space are W1 x1, rows [N1, N1 + N2) are W2 x2, both with K columns.
struct GemvPair {
  const float* x[2];
  const __nv_bfloat16* W[2];
  float* out[2];
  int64_t ldo[2];
  int N[2];
};

template <int NB>
__global__ void __launch_bounds__(32 * GEMV_WARPS)
    decode_gemv_kernel(const GemvPair pr, int64_t ldx, int64_t ldw, int B, int K) {
  pdl_enter();
  extern __shared__ float xs[];  // (products) x B x K
  const int np = pr.N[1] > 0 ? 2 : 1;
  for (int i = threadIdx.x; i < np * B * K; i += blockDim.x) {
    const int p = i / (B * K), r = i - p * B * K;
    const int b = r / K, k = r - b * K;
    xs[i] = (p ? pr.x[1] : pr.x[0])[(int64_t)b * ldx + k];
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int rows = pr.N[0] + pr.N[1];
  for (int row = blockIdx.x * GEMV_WARPS + (threadIdx.x >> 5); row < rows; row += gridDim.x * GEMV_WARPS) {
    const int p = row < pr.N[0] ? 0 : 1;
    const int n = p ? row - pr.N[0] : row;
    const float* xp = xs + p * B * K;
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.f;
    const __nv_bfloat16* wr = (p ? pr.W[1] : pr.W[0]) + (int64_t)n * ldw;
    for (int k8 = lane * 8; k8 < K; k8 += 256) {
      const uint4 pk = *reinterpret_cast<const uint4*>(wr + k8);
      const uint32_t w4[4] = {pk.x, pk.y, pk.z, pk.w};
      float wv[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 h2;
        memcpy(&h2, &w4[j], 4);
        const float2 f = __bfloat1622float2(h2);
        wv[2 * j] = f.x;
        wv[2 * j + 1] = f.y;
      }
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (b < B) {
          const float4 x0 = *reinterpret_cast<const float4*>(xp + b * K + k8);
          const float4 x1 = *reinterpret_cast<const float4*>(xp + b * K + k8 + 4);
          acc[b] = fmaf(wv[0], x0.x, acc[b]);
          acc[b] = fmaf(wv[1], x0.y, acc[b]);
          acc[b] = fmaf(wv[2], x0.z, acc[b]);
          acc[b] = fmaf(wv[3], x0.w, acc[b]);
          acc[b] = fmaf(wv[4], x1.x, acc[b]);
          acc[b] = fmaf(wv[5], x1.y, acc[b]);
          acc[b] = fmaf(wv[6], x1.z, acc[b]);
          acc[b] = fmaf(wv[7], x1.w, acc[b]);
        }
      }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      float v = acc[b];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (b < B && lane == 0) (p ? pr.out[1] : pr.out[0])[(int64_t)b * (p ? pr.ldo[1] : pr.ldo[0]) + n] = v;
    }
  }
}

int decode_gemv_launch(const GemvPair& pr, int64_t ldx, int64_t ldw, int64_t B, int64_t K, cudaStream_t st) {
  const int np = pr.N[1] > 0 ? 2 : 1;
  const size_t smem = (size_t)np * B * K * sizeof(float);
  const int dev = current_device();
  const int64_t rows = (int64_t)pr.N[0] + pr.N[1];
  const int64_t grid = std::min<int64_t>(cdiv(rows, GEMV_WARPS), 4LL * (dev >= 0 ? sm_count(dev) : 148));
  auto kern = B <= 1 ? decode_gemv_kernel<1> : decode_gemv_kernel<GEMV_MAX_B>;
  if (smem > 48 * 1024)
    ULM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  return launch_pdl(kern, dim3((unsigned)grid), dim3(32 * GEMV_WARPS), smem, st, pr, ldx, ldw, (int)B, (int)K);
}

int decode_gemv(const float* x, int64_t ldx, const __nv_bfloat16* W, int64_t ldw, float* out, int64_t ldo,
                int64_t B, int64_t N, int64_t K, cudaStream_t st) {
  GemvPair pr{{x, nullptr}, {W, nullptr}, {out, nullptr}, {ldo, 0}, {(int)N, 0}};
  return decode_gemv_launch(pr, ldx, ldw, B, K, st);
}

// two products with the same K, x row stride and weight row stride in one launch
int decode_gemv2(const float* x1, const __nv_bfloat16* W1, float* out1, int64_t ldo1, int64_t N1, const float* x2,
                 const __nv_bfloat16* W2, float* out2, int64_t ldo2, int64_t N2, int64_t ldx, int64_t ldw, int64_t B,
                 int64_t K, cudaStream_t st) {
  GemvPair pr{{x1, x2}, {W1, W2}, {out1, out2}, {ldo1, ldo2}, {(int)N1, (int)N2}};
  return decode_gemv_launch(pr, ldx, ldw, B, K, st);
}

// fp32 decode GEMM for small batches in the FMA back end's in-order form (the fp32 mode's run.c
// order): one thread per output row n walks k from 0 with one fused multiply-add per term, so the
// results equal the tiled kernel's with k_in_order bit for bit; its weight row is read with 16-byte
// loads, the batch's x rows sit in shared memory (read as broadcasts).
template <int NB>
__global__ void __launch_bounds__(128)
    decode_gemv_f32_kernel(const float* __restrict__ x, int64_t ldx, const float* __restrict__ W, int64_t ldw,
                           float* __restrict__ out, int64_t ldo, int B, int N, int K) {
  pdl_enter();
  extern __shared__ float xs[];  // B x K
  for (int i = threadIdx.x; i < B * K; i += blockDim.x) {
    const int b = i / K, k = i - b * K;
    xs[i] = x[(int64_t)b * ldx + k];
  }
  __syncthreads();
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const float4* wr = reinterpret_cast<const float4*>(W + (int64_t)n * ldw);
  float acc[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b] = 0.f;
#pragma unroll 4
  for (int k4 = 0; k4 < K / 4; ++k4) {
    const float4 w4 = wr[k4];
    const int k = 4 * k4;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      if (b < B) {
        const float* xb = xs + b * K + k;
        acc[b] = fmaf(xb[0], w4.x, acc[b]);
        acc[b] = fmaf(xb[1], w4.y, acc[b]);
        acc[b] = fmaf(xb[2], w4.z, acc[b]);
        acc[b] = fmaf(xb[3], w4.w, acc[b]);
      }
    }
  }
#pragma unroll
  for (int b = 0; b < NB; ++b)
    if (b < B) out[(int64_t)b * ldo + n] = acc[b];
}

// Whether the small-batch fp32 path serves a decode GEMM (K % 4 == 0, 16-byte weight rows).
bool gemv_f32_ok(int64_t B, int64_t K, int64_t ldw, const void* W) {
  return B <= GEMV_MAX_B && K % 4 == 0 && ldw % 4 == 0 && is_aligned16(W) &&
         B * K * (int64_t)sizeof(float) <= 48 * 1024;
}

int decode_gemv_f32(const float* x, int64_t ldx, const float* W, int64_t ldw, float* out, int64_t ldo, int64_t B,
                    int64_t N, int64_t K, cudaStream_t st) {
  const size_t smem = (size_t)B * K * sizeof(float);
  auto kern = B <= 1 ? decode_gemv_f32_kernel<1> : decode_gemv_f32_kernel<GEMV_MAX_B>;
  return launch_pdl(kern, dim3((unsigned)cdiv(N, 128)), dim3(128), smem, st, x, ldx, W, ldw, out, ldo, (int)B, (int)N,
                    (int)K);
}

// Whether the small-batch path serves a bf16 decode GEMM (x fp32 rows of ldx, 16-byte weight rows).
bool gemv_ok(int64_t B, int64_t K, int64_t ldw, int64_t ldx, const void* x, const void* W) {
  return B <= GEMV_MAX_B && K % 8 == 0 && ldw % 8 == 0 && ldx % 4 == 0 && is_aligned16(x) && is_aligned16(W) &&
         B * K * (int64_t)sizeof(float) <= 200 * 1024;
}

}  // namespace ulm

namespace {

// C[b][n] = sum_k X[b][k] W[n][k] for the decode batch; fp32 FMA or bf16 tensor cores.
int decode_gemm(const void* X, int64_t ldx, const void* W, int64_t ldw, int wdt, float* out, int64_t ldo, int64_t B,
                int64_t N, int64_t K, cudaStream_t st) {
  Operand A{X, ldx, B * ldx, K, B, wdt, false};
  Operand Bw{W, ldw, N * ldw, K, N, wdt, false};
  GemmShape s{1, (int)B, (int)N, (int)K, CAUSAL_NONE};
  s.k_in_order = 1;  // fp32 weights: run.c's dot-product order
  GemmEpilogue e;
  e.kind = EPI_STORE;
  e.out_dtype = ULM_F32;
  e.out = out;
  e.ldo = ldo;
  e.out_bstride = B * ldo;
  e.g = nullptr;
  e.aux = nullptr;
  e.ld_aux = 0;
  e.aux_bstride = 0;
  e.tile_partial = nullptr;
  e.row_partial = nullptr;
  e.part_ld = 0;
  e.staged = 0;
  e.vec_ok = is_aligned16(out) && ldo % 4 == 0;
  return run_gemm(A, Bw, s, e, st);
}

}  // namespace

// ---- sampling (run.c sample, run.c:460-534) ---------------------------------------------------
// One CTA of SMP_THREADS per sequence.
// Order of the probabilities for top-p: descending value, ties by ascending index, encoded as the
// 64-bit key (float bits of p) << 32 | (~index); excluded entries have key 0.
constexpr int SMP_THREADS = 1024;
constexpr int SMP_MAX_V = 50000;  // probabilities of one sequence in shared memory (200 KB)

__device__ __forceinline__ uint64_t smp_key(float p, int i) {
  return ((uint64_t)__float_as_uint(p) << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)i);
}

// fixed-order block reductions over SMP_THREADS threads (scratch: 32 slots)
__device__ __forceinline__ float smp_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[wp] = v;
  __syncthreads();
  if (wp == 0) {
    v = red[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[32] = v;
  }
  __syncthreads();
  return red[32];
}

__device__ __forceinline__ float smp_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[wp] = v;
  __syncthreads();
  if (wp == 0) {
    v = red[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[32] = v;
  }
  __syncthreads();
  return red[32];
}

__device__ __forceinline__ uint64_t smp_max_u64(uint64_t v, uint64_t* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t u = __shfl_xor_sync(0xffffffffu, v, o);
    v = u > v ? u : v;
  }
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[wp] = v;
  __syncthreads();
  if (wp == 0) {
    v = red[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t u = __shfl_xor_sync(0xffffffffu, v, o);
      v = u > v ? u : v;
    }
    if (lane == 0) red[32] = v;
  }
  __syncthreads();
  return red[32];
}

// key of entry i (0 when excluded by the cutoff or past V)
__device__ __forceinline__ uint64_t smp_entry_key(const float* ps, int i, int V, float cutoff) {
  return (i < V && ps[i] >= cutoff) ? smp_key(ps[i], i) : 0ull;
}

// the largest key K in [lo, hi] with sum over entries with key >= K of p > thresh (hi is a key; the
// answer is an entry's key), or 0 when even the sum over [lo, ...] does not exceed thresh
__device__ uint64_t smp_search(const float* ps, int V, float cutoff, uint64_t lo, uint64_t hi, float thresh,
                               float* red) {
  uint64_t ans = 0;
  while (lo <= hi && hi != 0) {
    const uint64_t mid = lo + (hi - lo) / 2;
    float s = 0.f;
    for (int i = threadIdx.x; i < V; i += SMP_THREADS) s += smp_entry_key(ps, i, V, cutoff) >= mid ? ps[i] : 0.f;
    s = smp_sum(s, red);
    if (s > thresh) {
      ans = mid;
      lo = mid + 1;
    } else {
      if (mid == 0) break;
      hi = mid - 1;
    }
  }
  return ans;
}

// next_token[b] from logits[b] as run.c's sample() with temperature > 0: softmax(logits / T), a coin
// from the sequence's xorshift64* state (run.c random_f32), then multinomial over the index order
// (topp outside (0, 1)) or top-p over the probabilities sorted descending; x[b] <- emb[next_token].
// The V probabilities live in dynamic shared memory (entry i at ps[i], thread i % SMP_THREADS).
__global__ void __launch_bounds__(SMP_THREADS)
    decode_sample_kernel(const float* __restrict__ logits, int V, float temperature, float topp,
                         unsigned long long* __restrict__ rng, int* __restrict__ next_token,
                         const void* __restrict__ emb, int emb_bf16, int D, float* __restrict__ x) {
  pdl_enter();
  extern __shared__ float ps[];
  __shared__ float red[33];
  __shared__ uint64_t redk[33];
  __shared__ float coin_s;
  __shared__ int pick;
  const int b = blockIdx.x, tid = threadIdx.x;
  const float* lg = logits + (int64_t)b * V;
  float mx = -INFINITY;
  for (int i = tid; i < V; i += SMP_THREADS) {
    const float v = lg[i] / temperature;
    ps[i] = v;
    mx = fmaxf(mx, v);
  }
  mx = smp_max(mx, red);
  float s = 0.f;
  for (int i = tid; i < V; i += SMP_THREADS) {
    const float e = expf(ps[i] - mx);
    ps[i] = e;
    s += e;
  }
  s = smp_sum(s, red);
  for (int i = tid; i < V; i += SMP_THREADS) ps[i] = ps[i] / s;
  if (tid == 0) {
    // xorshift64* step and 24-bit uniform (the published generator run.c uses)
    unsigned long long st = rng[b];
    st ^= st >> 12;
    st ^= st << 25;
    st ^= st >> 27;
    rng[b] = st;
    const uint32_t u = (uint32_t)((st * 0x2545F4914F6CDD1Dull) >> 32);
    coin_s = (float)(u >> 8) / 16777216.0f;
    pick = V - 1;
  }
  __syncthreads();
  const float coin = coin_s;
  if (!(topp > 0.f && topp < 1.f)) {
    // multinomial in index order: first i with coin < cdf_i, chunks of SMP_THREADS entries scanned
    // in turn (run.c sample_mult)
    __shared__ float wtot[32];
    __shared__ int hit_idx;
    if (tid == 0) hit_idx = 0x7fffffff;
    const int lane = tid & 31, wp = tid >> 5;
    float base = 0.f;
    for (int c0 = 0; c0 < V; c0 += SMP_THREADS) {
      const int i = c0 + tid;
      float v = i < V ? ps[i] : 0.f;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      __syncthreads();
      if (lane == 31) wtot[wp] = v;
      __syncthreads();
      float off = base, tot = 0.f;
      for (int w2 = 0; w2 < 32; ++w2) {
        if (w2 < wp) off += wtot[w2];
        tot += wtot[w2];
      }
      const unsigned mask = __ballot_sync(0xffffffffu, i < V && coin < off + v);
      if (lane == 0 && mask) atomicMin(&hit_idx, c0 + wp * 32 + __ffs(mask) - 1);
      base += tot;
      __syncthreads();
      if (hit_idx != 0x7fffffff) break;
    }
    if (tid == 0 && hit_idx != 0x7fffffff) pick = hit_idx;
    __syncthreads();
  } else {
    const float cutoff = (1.0f - topp) / (float)(V - 1);
    uint64_t kmax = 0;
    for (int i = tid; i < V; i += SMP_THREADS) {
      const uint64_t k = smp_entry_key(ps, i, V, cutoff);
      kmax = k > kmax ? k : kmax;
    }
    kmax = smp_max_u64(kmax, redk);
    // the top-p prefix: the largest key whose cumulative mass (descending order) exceeds topp
    uint64_t k1 = smp_search(ps, V, cutoff, 1, kmax, topp, red);
    if (k1 == 0) k1 = 1;  // rounding: the whole candidate set
    float pk = 0.f;
    for (int i = tid; i < V; i += SMP_THREADS) pk += smp_entry_key(ps, i, V, cutoff) >= k1 ? ps[i] : 0.f;
    pk = smp_sum(pk, red);
    // the first entry (descending order) whose cumulative mass exceeds coin * pk
    const uint64_t k2 = smp_search(ps, V, cutoff, k1, kmax, coin * pk, red);
    const uint64_t kk = k2 ? k2 : k1;
    if (tid == 0) pick = (int)(0xFFFFFFFFu - (uint32_t)(kk & 0xFFFFFFFFull));
    __syncthreads();
  }
  const int tok = pick;
  if (tid == 0) next_token[b] = tok;
  for (int i = tid; i < D; i += blockDim.x) {
    const int64_t o = (int64_t)tok * D + i;
    x[(int64_t)b * D + i] = emb_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(emb)[o])
                                     : static_cast<const float*>(emb)[o];
  }
}

extern "C" int ulm_decode_prepare_block(const float* mu, const float* w, const float* lam, void* prior,
                                        int prior_dtype, int64_t D, int64_t M, void* stream) {
  ULM_REQUIRE(mu && w && lam && prior, "null pointer argument");
  ULM_REQUIRE(weight_dtype_ok(prior_dtype), "prior_dtype must be ULM_F32 or ULM_BF16");
  ULM_REQUIRE(D > 0 && M > 0, "empty block");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  decode_prepare_kernel<<<(unsigned)std::min<int64_t>(cdiv(D * M, 256), 4 * 148), 256, 0, st>>>(
      mu, w, lam, prior, prior_dtype == ULM_BF16, (int)D, (int)M);
  ULM_LAUNCH_CHECK("decode_prepare_kernel");
  return ULM_OK;
}

extern "C" int ulm_decode_reset_block(const float* mu, const float* w, float* U, float* c, float* r_prev, float* buf,
                                      int64_t B, int64_t D, int64_t M, int64_t conv_size, void* stream) {
  ULM_REQUIRE(mu && w && U && c && r_prev && (buf || conv_size <= 1), "null pointer argument");
  ULM_REQUIRE(B > 0 && D > 0 && M > 0 && conv_size >= 1, "bad extents");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  decode_reset_kernel<<<(unsigned)std::min<int64_t>(cdiv(B * D * M, 256), 8 * 148), 256, 0, st>>>(
      mu, w, U, c, r_prev, buf, (int)B, (int)D, (int)M, (int)(conv_size - 1));
  ULM_LAUNCH_CHECK("decode_reset_kernel");
  return ULM_OK;
}

extern "C" int ulm_decode_block_step(float* x, const float* norm_w, const float* conv_w, const void* key_w,
                                     const float* key_b, const void* val_w, const void* prior, int weight_dtype,
                                     const float* w, const float* lam, const float* eps, float* U, float* c,
                                     float* r_prev, float* buf, void* work, int64_t B, int64_t D, int64_t M,
                                     int64_t conv_size, float norm_eps, void* stream) {
  ULM_REQUIRE(x && norm_w && conv_w && key_w && key_b && val_w && prior && w && lam && eps && U && c && r_prev &&
                  work,
              "null pointer argument");
  ULM_REQUIRE(weight_dtype_ok(weight_dtype), "weight_dtype must be ULM_F32 or ULM_BF16");
  ULM_REQUIRE(B > 0 && D > 0 && M > 0 && conv_size >= 1, "bad extents");
  ULM_REQUIRE(M % 4 == 0, "decode needs M %% 4 == 0 (16-byte state rows), got %lld", (long long)M);
  ULM_REQUIRE(is_aligned16(U) && is_aligned16(r_prev) && is_aligned16(prior), "state / prior must be 16-byte aligned");
  ULM_REQUIRE(B * D < (1ll << 31) / 8, "batch x dim too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf = weight_dtype == ULM_BF16;
  const int64_t ldo = ulm_operand_ld(D);
  // workspace: h, u, v (B x D fp32), a, r_old, q (B x M fp32), bf16 copies of h and u (B x ldo),
  // each piece 256-byte aligned
  char* wp = static_cast<char*>(work);
  auto take = [&](int64_t bytes) {
    char* p = wp;
    wp += (bytes + 255) / 256 * 256;
    return p;
  };
  float* h = reinterpret_cast<float*>(take(B * D * 4));
  float* u = reinterpret_cast<float*>(take(B * D * 4));
  float* v = reinterpret_cast<float*>(take(B * D * 4));
  float* a = reinterpret_cast<float*>(take(B * M * 4));
  float* r_old = reinterpret_cast<float*>(take(B * M * 4));  // the step's incoming r_prev
  float* q = reinterpret_cast<float*>(take(B * M * 4));
  __nv_bfloat16* hop = reinterpret_cast<__nv_bfloat16*>(take(B * ldo * 2));
  __nv_bfloat16* uop = reinterpret_cast<__nv_bfloat16*>(take(B * ldo * 2));
  if (int rc = launch_pdl(decode_prologue_kernel, dim3((unsigned)B), dim3(dec_row_threads(B)), 0, st, x, norm_w,
                          conv_w, buf, h, u, bf ? hop : nullptr, bf ? uop : nullptr, ldo, (int)D, (int)conv_size,
                          norm_eps))
    return rc;
  if (bf) {
    if (gemv_ok(B, D, D, D, u, key_w) && gemv_ok(B, D, D, D, h, val_w) && 2 * B * D * 4 <= 200 * 1024) {
      // a = u K^T and v = h W_v^T in one launch
      if (int rc = decode_gemv2(u, static_cast<const __nv_bfloat16*>(key_w), a, M, M, h,
                                static_cast<const __nv_bfloat16*>(val_w), v, D, D, D, D, B, D, st))
        return rc;
    } else {
      if (int rc = decode_gemm(uop, ldo, key_w, D, ULM_BF16, a, M, B, M, D, st)) return rc;
      if (int rc = decode_gemm(hop, ldo, val_w, D, ULM_BF16, v, D, B, D, D, st)) return rc;
    }
  } else {
    if (gemv_f32_ok(B, D, D, key_w) && gemv_f32_ok(B, D, D, val_w)) {
      const float* kwf = static_cast<const float*>(key_w);
      const float* vwf = static_cast<const float*>(val_w);
      if (int rc = decode_gemv_f32(u, D, kwf, D, a, M, B, M, D, st)) return rc;
      if (int rc = decode_gemv_f32(h, D, vwf, D, v, D, B, D, D, st)) return rc;
    } else {
      if (int rc = decode_gemm(u, D, key_w, D, ULM_F32, a, M, B, M, D, st)) return rc;
      if (int rc = decode_gemm(h, D, val_w, D, ULM_F32, v, D, B, D, D, st)) return rc;
    }
  }
  if (int rc = launch_pdl(decode_address_kernel, dim3((unsigned)B), dim3(dec_row_threads(B)), 0, st, a, key_b, w, lam,
                          eps, c, r_prev, r_old, q, (int)M))
    return rc;
  const int warps = DEC_THREADS / 32;
  ULM_REQUIRE((B * D) % warps == 0, "B*D must be a multiple of %d", warps);
  // warps per state row: enough rows' loads in flight to cover the SMs at small batches
  int S = 1;
  while (S < warps && B * D * S < 16 * 148 && (int64_t)S * 128 < M) S *= 2;
  const unsigned blocks = (unsigned)(B * D * S / warps);
  auto launch = [&](auto kern, const auto* pr) {
    return launch_pdl(kern, dim3(blocks), dim3(DEC_THREADS), 0, st, U, pr, v, r_old, q, lam, x, (int)D, (int)M);
  };
  const auto* pb = static_cast<const __nv_bfloat16*>(prior);
  const auto* pf = static_cast<const float*>(prior);
  int rc_state;
  if (S == 1)
    rc_state = bf ? launch(decode_state_kernel<__nv_bfloat16, 1>, pb) : launch(decode_state_kernel<float, 1>, pf);
  else if (S == 2)
    rc_state = bf ? launch(decode_state_kernel<__nv_bfloat16, 2>, pb) : launch(decode_state_kernel<float, 2>, pf);
  else if (S == 4)
    rc_state = bf ? launch(decode_state_kernel<__nv_bfloat16, 4>, pb) : launch(decode_state_kernel<float, 4>, pf);
  else
    rc_state = bf ? launch(decode_state_kernel<__nv_bfloat16, 8>, pb) : launch(decode_state_kernel<float, 8>, pf);
  return rc_state;
}

extern "C" int64_t ulm_decode_block_work_bytes(int64_t B, int64_t D, int64_t M) {
  auto al = [](int64_t n) { return (n + 255) / 256 * 256; };
  return 3 * al(B * D * 4) + 3 * al(B * M * 4) + 2 * al(B * ulm_operand_ld(D) * 2);
}

extern "C" int ulm_decode_embed(const int* tokens, const void* emb, int emb_dtype, float* x, int64_t B, int64_t D,
                                void* stream) {
  ULM_REQUIRE(tokens && emb && x, "null pointer argument");
  ULM_REQUIRE(weight_dtype_ok(emb_dtype), "emb_dtype must be ULM_F32 or ULM_BF16");
  if (int rc = launch_pdl(decode_embed_kernel, dim3((unsigned)B), dim3(128), 0, static_cast<cudaStream_t>(stream),
                          tokens, emb, emb_dtype == ULM_BF16, (int)D, x))
    return rc;
  return ULM_OK;
}

extern "C" int ulm_decode_head(float* x, const float* norm_w, const void* cls_w, const void* emb, int weight_dtype,
                               float* logits, int* next_token, void* work, int64_t B, int64_t D, int64_t V,
                               float norm_eps, void* stream) {
  ULM_REQUIRE(x && norm_w && cls_w && emb && logits && next_token && work, "null pointer argument");
  ULM_REQUIRE(weight_dtype_ok(weight_dtype), "weight_dtype must be ULM_F32 or ULM_BF16");
  ULM_REQUIRE(B > 0 && D > 0 && V > 0, "bad extents");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf = weight_dtype == ULM_BF16;
  const int64_t ldo = ulm_operand_ld(D);
  float* xn = static_cast<float*>(work);
  __nv_bfloat16* xop = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(work) + (B * D * 4 + 255) / 256 * 256);
  if (int rc = launch_pdl(decode_final_norm_kernel, dim3((unsigned)B), dim3(dec_row_threads(B)), 0, st, x, norm_w, xn,
                          bf ? xop : nullptr, ldo, (int)D, norm_eps))
    return rc;
  if (bf && gemv_ok(B, D, D, D, xn, cls_w)) {
    if (int rc = decode_gemv(xn, D, static_cast<const __nv_bfloat16*>(cls_w), D, logits, V, B, V, D, st)) return rc;
  } else if (bf) {
    if (int rc = decode_gemm(xop, ldo, cls_w, D, ULM_BF16, logits, V, B, V, D, st)) return rc;
  } else {
    if (gemv_f32_ok(B, D, D, cls_w)) {
      if (int rc = decode_gemv_f32(xn, D, static_cast<const float*>(cls_w), D, logits, V, B, V, D, st)) return rc;
    } else if (int rc = decode_gemm(xn, D, cls_w, D, ULM_F32, logits, V, B, V, D, st)) {
      return rc;
    }
  }
  if (int rc = launch_pdl(decode_argmax_embed_kernel, dim3((unsigned)B), dim3(dec_row_threads(B)), 0, st, logits, V,
                          (int)V, emb, bf, (int)D, next_token, x))
    return rc;
  return ULM_OK;
}

extern "C" int64_t ulm_decode_head_work_bytes(int64_t B, int64_t D) {
  return (B * D * 4 + 255) / 256 * 256 + (B * ulm_operand_ld(D) * 2 + 255) / 256 * 256;
}

extern "C" int ulm_decode_sample(const float* logits, int64_t B, int64_t V, float temperature, float topp,
                                 unsigned long long* rng_state, int* next_token, const void* emb, int emb_dtype,
                                 float* x, int64_t D, void* stream) {
  ULM_REQUIRE(logits && rng_state && next_token && emb && x, "null pointer argument");
  ULM_REQUIRE(weight_dtype_ok(emb_dtype), "emb_dtype must be ULM_F32 or ULM_BF16");
  ULM_REQUIRE(B > 0 && V > 1 && D > 0 && B < (1 << 30), "bad extents");
  ULM_REQUIRE(V <= SMP_MAX_V, "vocabulary larger than %d", SMP_MAX_V);
  ULM_REQUIRE(temperature > 0.f, "temperature must be > 0 (0 is the greedy pick of ulm_decode_head)");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t smem = (size_t)V * sizeof(float);
  ULM_CUDA_TRY(cudaFuncSetAttribute(decode_sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  if (int rc = launch_pdl(decode_sample_kernel, dim3((unsigned)B), dim3(SMP_THREADS), smem, st, logits, (int)V,
                          temperature, topp, rng_state, next_token, emb, emb_dtype == ULM_BF16 ? 1 : 0, (int)D, x))
    return rc;
  return ULM_OK;
}
