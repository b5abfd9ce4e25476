/*
 * ulm_b200.h - C ABI of the B200 (sm_100a) fast-memory library for UnifiedLM.
 *
 * Every entry point takes plain device pointers, element counts / strides in elements, and a
 * CUDA stream passed as `void*` (NULL = legacy default stream). Work is enqueued on that stream
 * and the call returns without synchronising. Outputs are written into caller-owned buffers;
 * nothing here allocates device memory unless a comment says otherwise. The return value is a
 * ulm_status; on failure `ulm_last_error()` returns a message for the calling thread.
 *
 * Tensors are row-major. "(B,T,M) ld" means element [b][t][m] lives at
 * base + (b*T + t)*ld + m, with ld >= M. Scalars that the reference keeps on the device (the log
 * decay g) are passed as device pointers so no call needs a host synchronisation.
 *
 * Reference interfaces replaced (file:line in ruhai-lin/unifiedlm.c):
 *   kernel.py:199-238  UnifiedMemory / unified_memory      -> ulm_memory_fwd, ulm_memory_bwd
 *   kernel.py:109-136  _fwd_stats_kernel                     -> ulm_memory_stats_fwd
 *   kernel.py:139-180  _bwd_stats_kernel + shift-add (:232)  -> ulm_memory_stats_bwd
 *   kernel.py:51-72    _la_attn_kernel (decayed chunk scores) -> ulm_decayed_scores
 *   kernel.py:23-48,
 *   kernel.py:75-101   _la_state / _la_out (apply scores)     -> ulm_causal_apply
 *   model.py:61-79     conv + UnifiedBlock.code (address)     -> ulm_address_fwd, ulm_address_bwd
 *   model.py:84-85     unified_memory + mu(q w) + residual    -> ulm_memory_combine_fwd, _bwd
 *   model.py:72,75,84  log_eps / log_w / log_rate transforms   -> ulm_block_scalars_fwd, _bwd
 *   model.py:88-111,   UnifiedBlock.init_state / step, and
 *   run.c:121-265      run.c reset_state / forward            -> ulm_decode_* (batched)
 *   run.c:460-534      run.c sample (argmax / mult / top-p)   -> ulm_decode_head, ulm_decode_sample
 *   model.py:153-157   output Linear + F.cross_entropy        -> ulm_lm_head_loss_fwd, _bwd
 */
#ifndef ULM_B200_H
#define ULM_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
enum {
  ULM_OK = 0,
  ULM_ERR_INVALID = 1,     /* bad argument: shape, stride, alignment, null pointer, dtype */
  ULM_ERR_CUDA = 2,        /* a CUDA runtime / driver call failed */
  ULM_ERR_UNSUPPORTED = 3, /* the device is not sm_100 or a required driver entry point is missing */
  ULM_ERR_DEVICE = 4       /* a kernel recorded a device-side error (see ulm_device_error) */
};

/* element types */
enum { ULM_F32 = 0, ULM_BF16 = 1 };

/* contraction precision of the chunk products:
 *   ULM_PREC_BF16: bf16 operands on the tcgen05 tensor cores, fp32 accumulation (the reference's
 *                  choice, kernel.py:205, 219);
 *   ULM_PREC_FP32: fp32 operands and fp32 FMA accumulation (the 1e-5 parity mode). */
enum { ULM_PREC_BF16 = 0, ULM_PREC_FP32 = 1 };

/* ---- library ------------------------------------------------------------------------------ */

/* Message describing the last failure on the calling thread ("" if none). */
const char* ulm_last_error(void);

/* ABI version of this library. */
int ulm_version(void);

/* Synchronises the current device, then reads and clears its device-side error flag: *site = 0
 * when no kernel gave up a bounded wait, otherwise the site code of the first one. */
int ulm_device_error(int* site);

/* ---- fast-memory statistics (kernel.py:109-136, 139-180) ----------------------------------- */

/* Forward slot statistics, per batch row b and slot a (lam = exp(*g)):
 *   k_t = r_{t-1} (k_0 = 0),  c_t = w + sum_{s<=t} lam^(t-s) k_s,  q_t = r_t / c_t.
 * r, q, c: (B,T,M) fp32 with row stride M. qop, kop: (B,T,M) copies of q and k in `op_dtype`
 * (ULM_BF16 for the tensor-core products, ULM_F32 for the fp32 mode) with row stride ld_op >= M.
 * w: (M,) fp32. g: device fp32 scalar. c may be NULL when ulm_memory_needs_c(T, M) is 0 (then the
 * backward rebuilds it from r). */
int ulm_memory_stats_fwd(const float* r, const float* w, const float* g, float* q, float* c, void* qop,
                         void* kop, int op_dtype, int64_t ld_op, int64_t B, int64_t T, int64_t M,
                         void* stream);

/* Backward of the statistics, walking time in reverse. Inputs: dqf = gradient reaching q through
 * the fast read, dq_out = gradient on the q output (may be NULL), dk = gradient reaching k through
 * the fast read, and the saved q, c, r. Outputs:
 *   dr  (B,T,M) fp32 : dq/c plus the shifted write-address gradient dk_total[t+1]
 *   dw  (M,)    fp32 : sum over b,t of dc                          (overwritten, not accumulated)
 *   dg  (1,)    fp32 : d/dg of the memory terms                    (overwritten)
 * `partial` is caller-provided scratch of ulm_memory_stats_bwd_scratch(B,T,M) bytes.
 * q and c may both be NULL when ulm_memory_needs_c(T, M) is 0 and every array is 16-byte aligned:
 * the kernel then rebuilds them from r with the forward scan (saves reading two fp32 arrays).
 * The sums over batch rows and positions run in a fixed order: results are deterministic. */
int ulm_memory_stats_bwd(const float* dqf, const float* dq_out, const float* dk, const float* q, const float* c,
                         const float* r, const float* w, const float* g, float* dr, float* dw, float* dg,
                         void* partial, int64_t B, int64_t T, int64_t M, void* stream);

int64_t ulm_memory_stats_bwd_scratch(int64_t B, int64_t T, int64_t M);

/* 1 if the statistics backward needs the saved c for a (T, M) problem, 0 if it can rebuild q and c
 * from r (the TMA-staged scans with 128-position CTAs: M % 4 == 0 and T <= 1024). */
int ulm_memory_needs_c(int64_t T, int64_t M);

/* Size of the scratch block built into the library for ulm_memory_stats_bwd_noalloc (per device). */
#define ULM_NOALLOC_SCRATCH_BYTES (8u << 20)

/* Same computation and results as ulm_memory_stats_bwd, for callers that cannot allocate device
 * memory when they call it (a serving runtime that reserves all of HBM for its own pool at start-up,
 * a plugin host that owns every device allocation). No reference counterpart: the reference
 * allocates its temporaries with torch (kernel.py:225-227).
 * It allocates nothing: its scratch is an 8 MiB block compiled into the library, which every GPU
 * that loads the library holds until the process exits. Limit: the scratch it needs, about
 * 34 * B * M bytes, must fit that block, so B * M up to about 246,000 (B=16 with M=2048 uses 1.1 MiB;
 * B=64 with M=3840 is about the largest); larger calls fail with ULM_ERR_INVALID and a message
 * (calls with B, T or M zero only zero dw and dg, as ulm_memory_stats_bwd does). Each call outside
 * stream capture looks up the block's device address (cudaGetSymbolAddress) in the calling
 * thread's current context, so contexts a host creates itself and the primary context after a
 * cudaDeviceReset each get their own address; a call during stream capture reuses the address an
 * earlier call in the same context recorded, so make one call in each context before capturing.
 * All calls share the one block, so calls that overlap on the GPU (different streams, no ordering
 * between them) race and must be avoided; calls on one stream are safe. */
int ulm_memory_stats_bwd_noalloc(const float* dqf, const float* dq_out, const float* dk, const float* q,
                                 const float* c, const float* r, const float* w, const float* g, float* dr,
                                 float* dw, float* dg, int64_t B, int64_t T, int64_t M, void* stream);

/* ---- the chunk products -------------------------------------------------------------------- */

/* Decayed causal scores over the whole sequence (the reference's intra-chunk matrix A_n,
 * kernel.py:51-72, extended across chunks):
 *   P[b][t][s] = lam^(t-s) * sum_k a[b][t][k] * bb[b][s][k]   for s <= t, and 0 for s > t
 * a, bb: (B,T,K) with row strides lda, ldb; P: (B,T,T) with row stride ldp. Only the tiles on or
 * below the diagonal are written (128 x 128 granularity in bf16 precision).
 * prec = ULM_PREC_BF16: a, bb, P are bf16; lda, ldb, ldp multiples of 8; 16-byte aligned bases.
 * prec = ULM_PREC_FP32: a, bb, P are fp32. */
int ulm_decayed_scores(const void* a, int64_t lda, const void* bb, int64_t ldb, void* P, int64_t ldp,
                       const float* g, int64_t B, int64_t T, int64_t K, int prec, void* stream);

/* Apply decayed scores to values (the products of kernel.py:75-101):
 *   transpose = 0 : o[b][t][v] = sum_{s<=t} P[b][t][s] * c[b][s][v]     (forward read)
 *   transpose = 1 : o[b][s][v] = sum_{t>=s} P[b][t][s] * c[b][t][v]     (time-reversed read)
 * P: (B,T,T) ldp; c: (B,T,V) ldc; o: (B,T,V) ldo with element type o_dtype (ULM_F32 / ULM_BF16).
 * Operand types and alignment follow `prec` as in ulm_decayed_scores. */
int ulm_causal_apply(const void* P, int64_t ldp, const void* c, int64_t ldc, void* o, int64_t ldo, int o_dtype,
                     int transpose, int64_t B, int64_t T, int64_t V, int prec, void* stream);

/* ---- the whole operator (kernel.py:199-238) ---------------------------------------------------- */

/* Padded row stride used for the operand copies of a length-n row (multiple of 8 elements). */
int64_t ulm_operand_ld(int64_t n);

/* Library-wide choice for bf16 products with M, N >= 256: 1 (default) runs them on CTA pairs with the
 * 2-SM MMA (256 x 256 tiles), 0 on single CTAs (128 x 256 tiles). Returns the previous setting.
 * Both compute the same products; the switch exists for comparisons and tuning. */
int ulm_set_gemm_pairs(int enable);

/* Library-wide epilogue layout of the bf16 products: 0 = each thread stores its output row
 * segment directly; 1 (default) = each epilogue warp stages 32-row x 128-byte chunks in shared
 * memory and writes them with TMA tensor stores. Both compute the same values. Returns the
 * previous mode, or -1 (no change) for an unknown mode. */
int ulm_set_epilogue_mode(int mode);

/* Library-wide choice of the slot-statistics scan kernels for T <= 1024: 1 (default) = persistent
 * clusters that walk (batch row, 32-slot block) items with the next item's tiles loading while the
 * current one is scanned; 0 = one cluster per item. Both compute the same values; they add the
 * per-warp partial sums in different groupings, so results agree to fp32 rounding. Returns the
 * previous mode, or -1 (no change) for an unknown mode. */
int ulm_set_scan_mode(int mode);

/* Library-wide switch of programmatic dependent launch: 1 (default) lets each kernel of the library
 * be scheduled while the previous kernel on its stream finishes (it waits for that kernel's results
 * on the device before touching memory); 0 launches every kernel after its predecessor has
 * completed. Results do not depend on it. Returns the previous setting. */
int ulm_set_pdl(int enable);

/* Form of the fast read's products (replaces the reference's fixed chunk length, kernel.py:20, 183-196).
 * Whole-sequence form: the decayed T x T scores and causal reads. Chunk-carry form with chunk length
 * C: a carry product walks the chunks with the (M x D) state in the tensor cores' accumulator and
 * writes one state per chunk boundary (the reference writes them for 64-token chunks, kernel.py:23-48),
 * an inter-chunk read against those states, and the whole-sequence products inside each chunk.
 * ulm_memory_chunk_len returns the chunk length the operator entry points use for (T, M, D, prec),
 * 0 for the whole-sequence form, -1 for bad arguments. Automatic choice (mode -1, default): for
 * ULM_PREC_BF16 the largest C in {1024, 512, 256} that divides T into at least two chunks, for
 * ULM_PREC_FP32 C = 64, where T (M + D) > 1.25 (4 M D + 2 C (M + D)) (the whole-sequence form's
 * flops per token against the chunked form's, with a margin for the chunked form's extra passes;
 * on B200 the chunked form wins at T = 8192 at the 42M and 110M widths, loses at T <= 4096).
 * ulm_set_chunk_mode: -1 automatic, 0 always the whole-sequence form, C > 0 (a multiple of 64, at
 * most 4096) that chunk length wherever T is a multiple of C with at least two chunks. Returns the
 * previous mode, or -2 (no change) for a bad mode. Buffers sized with ulm_memory_saved_bytes /
 * ulm_memory_bwd_work_bytes belong to the mode they were sized under. */
int ulm_set_chunk_mode(int mode);
int ulm_memory_chunk_len(int64_t T, int64_t M, int64_t D, int prec);
/* Bytes of the fast read's saved buffer (the `P` argument of the operator forwards) and of the
 * backward's work buffer (the `dS` argument of the operator backwards); -1 for bad arguments. */
int64_t ulm_memory_saved_bytes(int64_t B, int64_t T, int64_t M, int64_t D, int prec);
int64_t ulm_memory_bwd_work_bytes(int64_t B, int64_t T, int64_t M, int64_t D, int prec);

/* Forward of unified_memory(r, v, g, w) -> (q, fast).
 * Inputs : r (B,T,M) fp32; v (B,T,D) of type v_dtype, row stride D; g device scalar; w (M,) fp32.
 * den: NULL when r holds the read addresses; otherwise r holds their unnormalised form z
 * (ulm_address_fwd with normalize = 0) and den (B*T,) fp32 the row denominators, r = z / den,
 * applied as the rows are loaded.
 * Outputs: q (B,T,M) fp32; fast (B,T,D) of type v_dtype.
 * Saved for the backward (caller-owned, element type = ULM_BF16 for ULM_PREC_BF16, ULM_F32 for
 * ULM_PREC_FP32): c (B,T,M) fp32, or NULL when ulm_memory_needs_c(T, M) is 0; qop, kop
 * (B,T,ulm_operand_ld(M)); vop (B,T,ulm_operand_ld(D)); P: the fast read's saved buffer,
 * ulm_memory_saved_bytes(B,T,M,D,prec) bytes, 256-byte aligned. In the whole-sequence form
 * (ulm_memory_chunk_len(T,M,D,prec) == 0) it holds the decayed scores (B,T,ulm_operand_ld(T));
 * in the chunk-carry form the intra-chunk scores, the chunk-boundary states and the inter-chunk
 * read. */
int ulm_memory_fwd(const float* r, const float* den, const void* v, int v_dtype, const float* g, const float* w,
                   float* q, void* fast, float* c, void* qop, void* kop, void* vop, void* P, int64_t B, int64_t T,
                   int64_t M, int64_t D, int prec, void* stream);

/* Backward of unified_memory. dq_out may be NULL; dfast (B,T,D) of type do_dtype; r and den as
 * given to ulm_memory_fwd. Workspace buffers (caller-owned): doop (B,T,ulm_operand_ld(D)) in the
 * operand type, dS of ulm_memory_bwd_work_bytes(B,T,M,D,prec) bytes (256-byte aligned; the score
 * gradient (B,T,ulm_operand_ld(T)) in the whole-sequence form), dqf and dk (B,T,M) fp32, `partial`
 * of ulm_memory_stats_bwd_scratch bytes.
 * Outputs: dr (B,T,M) fp32 (the gradient of the normalised addresses in both forms), dv (B,T,D)
 * of type do_dtype, dg (1,) fp32, dw (M,) fp32. */
int ulm_memory_bwd(const float* dq_out, const void* dfast, int do_dtype, const float* r, const float* den,
                   const float* g, const float* w, const float* q, const float* c, const void* qop, const void* kop,
                   const void* vop, const void* P, void* doop, void* dS, float* dqf, float* dk, void* partial,
                   float* dr, void* dv, float* dg, float* dw, int64_t B, int64_t T, int64_t M, int64_t D,
                   int prec, void* stream);

/* ---- the block's combine fused into the fast memory (model.py:84-85) ------------------------- */

/* The block's learned scalars from their log parameters (model.py:72, 75, 84), the reference's
 * expressions in fp32: w (M,) = exp(clamp(log_w, -7, 12)), eps = exp(clamp(log_eps, -10, 10)) and
 * g = -exp(log_rate) (the log decay), one launch; log_eps, log_rate, eps and g are single device
 * floats. */
int ulm_block_scalars_fwd(const float* log_w, const float* log_eps, const float* log_rate, float* w, float* eps,
                          float* g, int64_t M, void* stream);
/* Backward of ulm_block_scalars_fwd, as autograd of those expressions gives it: dlog_w = dw * w where
 * -7 <= log_w <= 12 (else 0), dlog_eps = deps * eps where -10 <= log_eps <= 10 (else 0),
 * dlog_rate = dg * g; w, eps and g are the forward's outputs. One launch. */
int ulm_block_scalars_bwd(const float* log_w, const float* log_eps, const float* w, const float* eps, const float* g,
                          const float* dw, const float* deps, const float* dg, float* dlog_w, float* dlog_eps,
                          float* dlog_rate, int64_t M, void* stream);

/* y = x + mu(q * w) + fast, (q, fast) = unified_memory(r, v, g, w): UnifiedBlock.forward's last
 * line (model.py:85, dropout off) with the combine's product mu(q w) accumulated in the same
 * tensor-core tiles as the fast read. Inputs as ulm_memory_fwd plus mu (D,M) fp32 (the `mu`
 * Linear's weight) and x (B,T,D) of x_dtype; y (B,T,D) of x_dtype. q (B,T,M) fp32 may be NULL when
 * c is NULL (the fp32 copy of q is then not written). Saved / scratch as ulm_memory_fwd plus wmu
 * (M, ulm_operand_ld(D)) in the operand type. */
int ulm_memory_combine_fwd(const float* r, const float* den, const void* v, int v_dtype, const float* g,
                           const float* w, const float* mu, const void* x, int x_dtype, void* y, float* q, float* c,
                           void* qop, void* kop, void* vop, void* P, void* wmu, int64_t B, int64_t T, int64_t M,
                           int64_t D, int prec, void* stream);

/* Backward of ulm_memory_combine_fwd from dy (B,T,D) of dy_dtype (dx = dy is the caller's). Saved
 * tensors and workspaces as ulm_memory_bwd plus mw (D, ulm_operand_ld(M)) in the operand type and
 * gpart of ulm_combine_grad_scratch bytes. Outputs: dr (B,T,M) fp32 (gradient of the normalised
 * addresses), dv (B,T,D) of dv_dtype, dg (1,), dw (M,) (both the statistics' and the combine's
 * share), dmu (D,M) fp32. */
int ulm_memory_combine_bwd(const void* dy, int dy_dtype, const float* r, const float* den, const float* g,
                           const float* w, const float* mu, const float* q, const float* c, const void* qop,
                           const void* kop, const void* vop, const void* P, void* doop, void* dS, void* mw,
                           float* dqf, float* dk, void* partial, float* gpart, float* dr, void* dv, int dv_dtype,
                           float* dg, float* dw, float* dmu, int64_t B, int64_t T, int64_t M, int64_t D, int prec,
                           void* stream);

int64_t ulm_combine_grad_scratch(int64_t B, int64_t T, int64_t M, int64_t D);

/* ---- the addressing prologue (model.py:61-62, 70-72, 79) -------------------------------------- */

/* r = z / (eps + sum_m z), z = relu(u key_w^T + key_b)^2, u = causal depthwise conv(h).
 * h: (B,T,D) of h_dtype; conv_w: (D,conv_size) fp32 oldest -> newest; key_w: (M, ld_kw) in the
 * operand type of prec (bf16 for ULM_PREC_BF16, fp32 for ULM_PREC_FP32); key_b: (M,) fp32;
 * eps: device scalar. Outputs: den (B*T) fp32 = eps + sum z (saved), u_op (B*T, ld_u) in the
 * operand type (saved), and in r (B,T,M) fp32: the addresses when normalize = 1, or z when
 * normalize = 0 (the row sums then come from the key product's epilogue and no pass rewrites r;
 * ulm_memory_fwd / ulm_memory_bwd / ulm_address_bwd take the pair (z, den)). work: caller scratch
 * of ulm_address_fwd_work_bytes(B,T,M) bytes, needed only when normalize = 0 (may be NULL
 * otherwise). */
int ulm_address_fwd(const void* h, int h_dtype, const float* conv_w, int64_t conv_size, const void* key_w,
                    int64_t ld_kw, const float* key_b, const float* eps, float* r, float* den, int normalize,
                    void* work, void* u_op, int64_t ld_u, int64_t B, int64_t T, int64_t D, int64_t M, int prec,
                    void* stream);

int64_t ulm_address_fwd_work_bytes(int64_t B, int64_t T, int64_t M);

/* Backward of ulm_address_fwd from dr (B,T,M) fp32, the gradient of the normalised addresses:
 * dh (B,T,D) fp32, dconv_w (D,conv_size), dkey_w (M,D), dkey_b (M,) and deps (1,) fp32 (all
 * overwritten). r and den as ulm_address_fwd left them; normalized = the normalize flag it ran
 * with. work: caller scratch of ulm_address_bwd_work_bytes(B,T,D,M,prec) bytes. Column sums run in
 * a fixed order. */
int ulm_address_bwd(const float* dr, const float* r, const float* den, int normalized, const void* u_op,
                    int64_t ld_u, const void* h, int h_dtype, const float* conv_w, int64_t conv_size,
                    const void* key_w, int64_t ld_kw, float* dh, float* dconv_w, float* dkey_w, float* dkey_b,
                    float* deps, void* work, int64_t B, int64_t T, int64_t D, int64_t M, int prec, void* stream);

int64_t ulm_address_bwd_work_bytes(int64_t B, int64_t T, int64_t D, int64_t M, int prec);

/* ---- the language-model head with its cross-entropy loss (model.py:153-157) ------------------ */

/* loss = F.cross_entropy(h W^T, targets, ignore_index=-1) without writing the (N,V) logits.
 * h_op (N, ld_h) and w_op (V, ld_w): the final-normed hidden states and the classifier weight in
 * the operand type of prec (bf16 for ULM_PREC_BF16, fp32 for ULM_PREC_FP32); targets (N,) int64.
 * Outputs: lse (N,) fp32 (each row's logsumexp, saved for the backward), loss (1,) fp32 (mean over
 * the rows whose target is not -1; nan when there are none), count (1,) fp32 (that number of rows).
 * work: ulm_lm_head_work_bytes(N,V,D,prec) bytes, shared with the backward. */
int ulm_lm_head_loss_fwd(const void* h_op, int64_t ld_h, const void* w_op, int64_t ld_w, const int64_t* targets,
                         float* lse, float* loss, float* count, void* work, int64_t N, int64_t V, int64_t D,
                         int prec, void* stream);

/* Backward: dh (N,D) fp32 and dW (V,D) fp32 for the upstream gradient dloss (device scalar);
 * count and lse as the forward left them. The logits are recomputed. */
int ulm_lm_head_loss_bwd(const float* dloss, const float* count, const void* h_op, int64_t ld_h, const void* w_op,
                         int64_t ld_w, const int64_t* targets, const float* lse, float* dh, float* dw, void* work,
                         int64_t N, int64_t V, int64_t D, int prec, void* stream);

int64_t ulm_lm_head_work_bytes(int64_t N, int64_t V, int64_t D, int prec);

/* The path's whole backward for one block with unnormalised addresses z (ulm_address_fwd with
 * normalize = 0): ulm_memory_bwd(dq_out, dfast, .., r = z, den, ..) followed by
 * ulm_address_bwd(dr, z, den, normalized = 0, ..), in one call; same arguments and outputs as the
 * two calls (dr is written as there), and the same results. In one call the statistics' dw / dg
 * reductions overlap the address backward; all work is ordered on `stream` when it returns.
 * Replaces: the backward of UnifiedBlock.forward's read path, model.py:70-84 (kernel.py:216-233
 * and the prologue's autograd). */
int ulm_addressed_memory_bwd(const float* dq_out, const void* dfast, int do_dtype, const float* z, const float* den,
                             const float* g, const float* w, const float* q, const float* c, const void* qop,
                             const void* kop, const void* vop, const void* P, void* doop, void* dS, float* dqf,
                             float* dk, void* partial, float* dr, void* dv, float* dg, float* dw, const void* u_op,
                             int64_t ld_u, const void* h, int h_dtype, const float* conv_w, int64_t conv_size,
                             const void* key_w, int64_t ld_kw, float* dh, float* dconv_w, float* dkey_w,
                             float* dkey_b, float* deps, void* work, int64_t B, int64_t T, int64_t M, int64_t D,
                             int prec, void* stream);

/* The same for the fused combine: ulm_memory_combine_bwd followed by ulm_address_bwd (model.py:70-85
 * with dropout 0). */
int ulm_mixer_bwd(const void* dy, int dy_dtype, const float* z, const float* den, const float* g, const float* w,
                  const float* mu, const float* q, const float* c, const void* qop, const void* kop, const void* vop,
                  const void* P, void* doop, void* dS, void* mw, float* dqf, float* dk, void* partial, float* gpart,
                  float* dr, void* dv, int dv_dtype, float* dg, float* dw, float* dmu, const void* u_op,
                  int64_t ld_u, const void* h, int h_dtype, const float* conv_w, int64_t conv_size,
                  const void* key_w, int64_t ld_kw, float* dh, float* dconv_w, float* dkey_w, float* dkey_b,
                  float* deps, void* work, int64_t B, int64_t T, int64_t M, int64_t D, int prec, void* stream);

/* ---- RMSNorm and Linear of the block's input side (model.py:31-42, 65, 81) --------------------- */

/* y = round_x(x * rstd) * weight, rstd = 1 / sqrt(mean(x^2) + eps) per row, in fp32 (the reference's
 * RMSNorm.forward, model.py:31-42; round_x = rounding to x's type, the reference's type_as(x)).
 * x (rows, D) of x_dtype, weight (D,) fp32, y (rows, D) of y_dtype, rstd (rows,) fp32 (may be NULL;
 * the backward needs it). */
int ulm_rms_norm_fwd(const void* x, int x_dtype, const float* weight, void* y, int y_dtype, float* rstd,
                     int64_t rows, int64_t D, float eps, void* stream);
/* Backward of ulm_rms_norm_fwd from dy (rows, D) of dy_dtype: dx (rows, D) fp32, plus dx_add
 * (rows, D) fp32 when not NULL (the gradient the input receives along another path, such as a
 * residual connection, added as dx is written), dweight (D,) fp32 (overwritten; summed over rows in
 * a fixed order). work: ulm_rms_norm_bwd_work_bytes(rows, D) bytes. D * 32 bytes must fit the
 * backward's shared memory (D <= 6400). */
int ulm_rms_norm_bwd(const void* dy, int dy_dtype, const void* x, int x_dtype, const float* weight,
                     const float* rstd, float* dx, const float* dx_add, float* dweight, void* work, int64_t rows,
                     int64_t D, void* stream);
int64_t ulm_rms_norm_bwd_work_bytes(int64_t rows, int64_t D);

/* y = x W^T (nn.Linear without bias; UnifiedBlock.val, model.py:65, 81): x (N, K) of x_dtype, weight
 * (Nout, K) fp32, y (N, Nout) of y_dtype. Writes the operand copies x_op (N, ulm_operand_ld(K)) and
 * w_op (Nout, ulm_operand_ld(K)) (bf16 for ULM_PREC_BF16, fp32 for ULM_PREC_FP32), which the
 * backward reads. */
int ulm_linear_fwd(const void* x, int x_dtype, const float* weight, void* x_op, void* w_op, void* y, int y_dtype,
                   int64_t N, int64_t K, int64_t Nout, int prec, void* stream);
/* Backward of ulm_linear_fwd from dy (N, Nout) of dy_dtype: dx (N, K) fp32 = dy W (+ dx_add (N, K)
 * fp32 when not NULL, added in the product's epilogue), dw (Nout, K) fp32 = dy^T x (split over the
 * rows, partials summed in a fixed order). work: ulm_linear_bwd_work_bytes(N, K, Nout, prec) bytes;
 * dy is read in place when it is already an operand (the operand type, Nout a multiple of 8 and a
 * 16-byte aligned start), else copied into the front of work. */
int ulm_linear_bwd(const void* dy, int dy_dtype, const void* x_op, const void* w_op, float* dx, const float* dx_add,
                   float* dw, void* work, int64_t N, int64_t K, int64_t Nout, int prec, void* stream);
int64_t ulm_linear_bwd_work_bytes(int64_t N, int64_t K, int64_t Nout, int prec);

/* ---- batched recurrent decode (model.py:88-111, 164-175; run.c:121-265) --------------------- */

/* Per block, once per weight set: prior[d][m] = ((1 - lam) * mu[d][m]) * w[m], the constant part of
 * the state update (run.c:251), stored as prior_dtype. mu: (D,M) fp32; w: (M,) fp32; lam: device
 * scalar. */
int ulm_decode_prepare_block(const float* mu, const float* w, const float* lam, void* prior, int prior_dtype,
                             int64_t D, int64_t M, void* stream);

/* Per block, at the start of every sequence batch (UnifiedBlock.init_state, model.py:88-94;
 * run.c reset_state, run.c:121-138): U = mu * w (B,D,M), c = w (B,M), r_prev = 0 (B,M),
 * conv buffer = 0 (B,D,conv_size-1). */
int ulm_decode_reset_block(const float* mu, const float* w, float* U, float* c, float* r_prev, float* buf,
                           int64_t B, int64_t D, int64_t M, int64_t conv_size, void* stream);

/* One token through one UnifiedBlock for B sequences (UnifiedBlock.step, model.py:96-111; the block
 * body of run.c forward, run.c:203-260): x (B,D) fp32 is updated in place (residual). Weights:
 * norm_w (D), conv_w (D,conv_size) fp32 oldest -> newest, key_w (M,D), val_w (D,D) and prior (D,M)
 * in weight_dtype (ULM_F32: fp32 FMA contractions, run.c's operation order in the state update;
 * ULM_BF16: bf16 weights on the tensor cores), key_b and w (M) fp32, lam and eps device scalars.
 * State (fp32, updated in place): U (B,D,M), c (B,M), r_prev (B,M), buf (B,D,conv_size-1).
 * work: caller scratch of ulm_decode_block_work_bytes(B,D,M) bytes. M must be a multiple of 4. */
int ulm_decode_block_step(float* x, const float* norm_w, const float* conv_w, const void* key_w, const float* key_b,
                          const void* val_w, const void* prior, int weight_dtype, const float* w, const float* lam,
                          const float* eps, float* U, float* c, float* r_prev, float* buf, void* work, int64_t B,
                          int64_t D, int64_t M, int64_t conv_size, float norm_eps, void* stream);

int64_t ulm_decode_block_work_bytes(int64_t B, int64_t D, int64_t M);

/* x[b] = emb[tokens[b]] (B,D) fp32; emb (V,D) in emb_dtype; tokens int32 on the device. */
int ulm_decode_embed(const int* tokens, const void* emb, int emb_dtype, float* x, int64_t B, int64_t D,
                     void* stream);

/* Final RMSNorm, logits = norm(x) cls_w^T (B,V) fp32, greedy next token (first index of the
 * largest logit, run.c sample_argmax) into next_token (B,) int32, and x <- emb[next_token] ready for
 * the next step. work: ulm_decode_head_work_bytes(B,D) bytes. */
int ulm_decode_head(float* x, const float* norm_w, const void* cls_w, const void* emb, int weight_dtype,
                    float* logits, int* next_token, void* work, int64_t B, int64_t D, int64_t V, float norm_eps,
                    void* stream);

int64_t ulm_decode_head_work_bytes(int64_t B, int64_t D);

/* Parallel prefill of one block (replaces feeding a prompt through UnifiedBlock.step token by
 * token, model.py:96-111 / run.c:193-265): after the training-form forward of the block over T
 * prompt positions (z and den from ulm_address_fwd with normalize = 0; kop (B,T,ulm_operand_ld(M))
 * and vop (B,T,ulm_operand_ld(D)) the operand copies of ulm_memory_fwd / ulm_memory_combine_fwd;
 * h (B,T,D) of h_dtype the block's normalised input), writes the decode state that T steps would
 * leave: U (B,D,M) = w mu + sum_s lam^(T-1-s) v_s k_s^T (k_s = r_{s-1}; one carry product over a
 * single chunk of T positions, straight into the (D,M) layout), c (B,M) = the evidence mass after
 * position T-1 (step's update order), r_prev (B,M) = r_{T-1}, buf (B,D,conv_size-1) = the last
 * conv_size-1 rows of h, oldest first (zero before position 0). g = log(lam) and lam are device
 * scalars; mu (D,M), w (M,) fp32; work: ulm_decode_prefill_work_bytes(B,T,D,prec) bytes. */
int ulm_decode_prefill_block(const void* kop, const void* vop, const float* g, const float* lam, const float* z,
                             const float* den, const void* h, int h_dtype, const float* mu, const float* w, void* work,
                             float* U, float* c, float* r_prev, float* buf, int64_t B, int64_t T, int64_t D, int64_t M,
                             int64_t conv_size, int prec, void* stream);
int64_t ulm_decode_prefill_work_bytes(int64_t B, int64_t T, int64_t D, int prec);

/* run.c's sample() with temperature > 0 (run.c:460-534) for B sequences on the device:
 * softmax(logits[b] / temperature), a coin from the sequence's xorshift64* state rng_state[b]
 * (advanced in place, run.c random_f32), then the first index whose cumulative probability exceeds
 * the coin (topp <= 0 or >= 1, run.c sample_mult) or top-p sampling over the probabilities sorted
 * in descending order (run.c sample_topp; ties by ascending index). Writes next_token (B,) int32
 * and x[b] = emb[next_token[b]]. The sums are parallel reductions, so a coin within about 1e-7 of a
 * cumulative boundary can pick the neighbouring token where run.c's sequential sums would not.
 * logits (B,V) fp32, V <= 50000; emb (V,D) in emb_dtype; x (B,D) fp32. */
int ulm_decode_sample(const float* logits, int64_t B, int64_t V, float temperature, float topp,
                      unsigned long long* rng_state, int* next_token, const void* emb, int emb_dtype, float* x,
                      int64_t D, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ULM_B200_H */
