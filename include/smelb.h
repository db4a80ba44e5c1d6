/*
 * smelb — B200 (sm_100a) implementation of the SMEL FT MoE expert layer, C ABI.
 *
 * Conventions
 *   - All tensors are device pointers to row-major, contiguous storage. bf16 values are passed as `void*`.
 *   - `stream` is a cudaStream_t passed as `void*` (NULL = legacy default stream). Every call is stream-ordered and
 *     keeps no state between calls except a per-device 4-byte status word (see smelb_read_status).
 *   - Every function returns 0 on success or a negative SMELB_ERR_* code; smelb_last_error() gives the text.
 *   - Nothing here allocates memory except the per-device status word (4 bytes, on first use) — the caller owns and
 *     passes every buffer.
 *
 * Reference interfaces (paths relative to the smel-ft source tree) are cited per entry point.
 */
#ifndef SMELB_H
#define SMELB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SMELB_OK 0
#define SMELB_ERR_SHAPE (-1)
#define SMELB_ERR_DTYPE (-2)
#define SMELB_ERR_WORKSPACE (-3)
#define SMELB_ERR_TIMEOUT (-4)
#define SMELB_ERR_CUDA (-5)
#define SMELB_ERR_ARG (-6)

#define SMELB_ACT_SILU 0      /* moe.py:91-96 act("silu") */
#define SMELB_ACT_GELU_TANH 1 /* moe.py:91-96 act("gelu_tanh") */

/* Library version (major * 10000 + minor * 100 + patch). */
int smelb_version(void);

/* Copies the text of the last error of the calling thread into buf (NUL-terminated). Returns its length. */
int smelb_last_error(char* buf, size_t len);

/* Makes `device` (and its primary context) current for this library on the calling thread. Bindings call it with
 * the framework's current device before the other entry points (e.g. on autograd worker threads). */
int smelb_set_device(int device);

/* Synchronizes `device` and reads its status word: 0, or the code of the first device-side wait that gave up
 * (a pipeline barrier that was never satisfied) or of an out-of-range expert index. reset != 0 clears it. */
int smelb_read_status(int device, int* status, int reset);

/* As smelb_read_status, with the location of the first failure: words[0] code, words[1] block, words[2] tile,
 * words[3] k-block (-1 where not applicable). words has 4 entries. */
int smelb_read_status_detail(int device, int* words, int reset);

/* ---------------------------------------------------------------------------------------------------- int4 format
 * smel/quant.py:74-94 dequant_int4 / dequant_int4_torch: q uint8 [rows, k/2] (low nibble = even column),
 * scale/zero bf16 [rows, groups] -> out [rows, k], out = q * scale + zero computed in fp32 and rounded once to the
 * output type (bf16, or fp32 when out_fp32 != 0). */
int smelb_int4_dequant(const void* q, const void* scale, const void* zero, void* out, int64_t rows, int64_t k,
                       int64_t groups, int out_fp32, void* stream);

/* smel/quant.py:87-94 dequant_int4_torch: the same dequant with every operation in the output dtype, as torch runs
 * it: with a bf16 output the product q * scale is rounded to bf16 before zero is added, and the sum is rounded again
 * (two roundings; smelb_int4_dequant rounds once). With out_fp32 != 0 the two entry points agree. */
int smelb_int4_dequant_stepwise(const void* q, const void* scale, const void* zero, void* out, int64_t rows,
                                int64_t k, int64_t groups, int out_fp32, void* stream);

/* smel/pack.py:28-46 merge_experts / merge_mlp with smel/lora.py:31-36,52-56 delta(): out [rows, cols] =
 * w + (scale * B) @ A, the rank-r product in fp32 as a fused multiply-add chain over the rank (the order of the
 * reference's fp32 matmul), added to w in fp32 and rounded once to w's dtype (bf16, or fp32 when w_fp32 != 0).
 * B fp32 [rows, r], A fp32 [r, cols]; out may alias w. */
int smelb_lora_merge(const void* w, int w_fp32, int64_t rows, int64_t cols, const float* B, const float* A, int64_t r,
                     float scale, void* out, void* stream);

/* smel/quant.py:14-44 quantize_int4 with group = 64: w [rows, k] (bf16, or fp32 when w_fp32 != 0) -> q uint8
 * [rows, k/2] (low nibble = even column), scale / zero bf16 [rows, k/64]. Per group the [min, max] range is shrunk
 * towards its center by each of the n_clip factors in `clip` (host array, 1..8 entries, the reference's
 * clip_search) and the candidate with the smallest squared error is kept (the earlier one on ties). k % 64 == 0. */
int smelb_int4_quantize(const void* w, int w_fp32, int64_t rows, int64_t k, const float* clip, int n_clip, void* q,
                        void* scale, void* zero, void* stream);

/* smel/moe.py:35-55 Int4Experts: builds the (scale | zero << 16) uint32 pairs transposed to [nw, groups, rows],
 * the layout the fused expert GEMMs stage per k-block. scale/zero bf16 [nw, rows, groups]. */
int smelb_int4_pack_sz(const void* scale, const void* zero, uint32_t* sz_t, int64_t nw, int64_t rows,
                       int64_t groups, void* stream);

/* ---------------------------------------------------------------------------------------------------- routing
 * smel/moe.py:162-167 route (softmax / top-k / renorm part) and moe.py:178-180 (route_gemma4 tail):
 * logits bf16 [T, E] (row pitch ld elements) -> probs fp32 [T, E], topv [T, K] (bf16, or fp32 if topv_fp32),
 * topi int64 [T, K]. Ties in probs are broken towards the smaller expert id. per_expert_scale (bf16 [E]) may be NULL.
 * E <= 512, K <= 32. */
int smelb_router_topk(const void* logits, int64_t ld, int64_t T, int64_t E, int64_t K, float* probs, void* topv,
                      int topv_fp32, int64_t* topi, const void* per_expert_scale, void* stream);

/* Backward of smelb_router_topk: d topv -> d logits (bf16 [T, E], row pitch ld). */
int smelb_router_bwd(const void* dtopv, int dtopv_fp32, const float* probs, const int64_t* topi,
                     const void* per_expert_scale, int64_t T, int64_t E, int64_t K, void* dlogits, int64_t ld,
                     void* stream);

/* smel/moe.py:216-223 (routed_experts dispatch): stable counting sort of topi.reshape(-1).
 *   counts[E]    int32  tokens per expert                   (bincount)
 *   gcounts[E]   int32  rows of each expert's segment (counts, rounded up to `pad` for experts with sel_mask[e])
 *   offsets[E]   int32  first row of each expert's segment
 *   row_of[T*K]  int32  dispatch row of choice t*K+k
 *   src_of[max]  int32  choice of each dispatch row (-1 on padding rows); max = T*K + (#selected) * pad
 *   order[T*K]   int64  torch.argsort(topi.reshape(-1), stable=True)
 *   total[1]     int32  rows used
 * sel_mask (uint8 [E]) may be NULL (no padding). E <= 512. */
int smelb_dispatch_plan(const int64_t* topi, int64_t T, int64_t K, int64_t E, const uint8_t* sel_mask, int64_t pad,
                        int32_t* counts, int32_t* gcounts, int32_t* offsets, int32_t* row_of, int32_t* src_of,
                        int64_t* order, int32_t* total, void* stream);

/* The same plan computed by many CTAs (same outputs, bit for bit). workspace: int32 scratch of workspace_ints
 * elements (up to 148 * E are used; with fewer than 2 * E it falls back to the one-CTA plan). */
int smelb_dispatch_plan_ws(const int64_t* topi, int64_t T, int64_t K, int64_t E, const uint8_t* sel_mask,
                           int64_t pad, int32_t* counts, int32_t* gcounts, int32_t* offsets, int32_t* row_of,
                           int32_t* src_of, int64_t* order, int32_t* total, int32_t* workspace,
                           int64_t workspace_ints, void* stream);

/* xs[row] = x[src_of[row] / K] (zeros on padding rows) for rows < total[0]. x bf16 [T, H], xs bf16 [max_rows, H]. */
int smelb_gather_rows(const void* x, int64_t H, int64_t K, const int32_t* src_of, const int32_t* total,
                      int64_t max_rows, void* xs, void* stream);

/* smel/moe.py:248-252 combine: out[t] = bf16(sum_k fp32(y[row_of[t,k]]) * fp32(topv[t,k])), k in order. */
int smelb_combine_fwd(const void* y, const int32_t* row_of, const void* topv, int topv_fp32, int64_t T, int64_t K,
                      int64_t H, void* out, void* stream);

/* Backward of smelb_combine_fwd for rows r < total[0] (src_of[r] = choice t*K+k, -1 on padding rows):
 * dy[r] = bf16(g[t] * topv[t,k]) (zeros on padding rows) and dtopv[t,k] = sum_h g[t,h] * y[r,h] in fp32 (stored as
 * bf16, or fp32 if topv_fp32). dtopv may be NULL. The autograd of moe.py:248-252. */
int smelb_combine_bwd(const void* g, const void* y, const int32_t* src_of, const int32_t* total, int64_t max_rows,
                      const void* topv, int topv_fp32, int64_t K, int64_t H, void* dy, void* dtopv, void* stream);

/* Backward of smelb_gather_rows: dx[t] = bf16(sum_k fp32(dxs[row_of[t,k]])) in k order (the autograd of the
 * x[tok] gather, moe.py:221). */
int smelb_gather_rows_bwd(const void* dxs, const int32_t* row_of, int64_t T, int64_t K, int64_t H, void* dx,
                          void* stream);

/* ---------------------------------------------------------------------------------------------------- row norms
 * smel/norm.py rmsnorm / add_rmsnorm (torch form smel/layer_runner.py:110-130), bf16 rows [rows, C] (C % 8 == 0),
 * fp32 math, one rounding to bf16:
 *   h_add == NULL: y = x * rstd * w';  h_add != NULL: s_out = bf16(h_add + x), y = s_out * rstd * w'
 *   w' = 1 (w_mode 0, w may be NULL), w (1, Gemma 4) or 1 + w (2, Qwen3.5/3.6); rstd = rsqrt(mean(v^2) + eps).
 * post_scale (bf16 [C]) / post_mul (0: none) add the Gemma 4 router prologue of smel/moe.py:170-176 in its bf16
 * steps: y = bf16(bf16(bf16(v * rstd) * post_scale) * post_mul) (w_mode 0). rstd_out (fp32 [rows]) may be NULL. */
int smelb_rmsnorm_fwd(const void* x, const void* h_add, const void* w, int w_mode, const void* post_scale,
                      float post_mul, float eps, int64_t rows, int64_t C, void* s_out, void* y, float* rstd_out,
                      void* stream);

/* Backward of smelb_rmsnorm_fwd with frozen weights: dx = rstd * (g - xhat * mean(g * xhat)) + ds, g = dy * w'
 * (through the post chain's bf16 steps when given), xhat = x * rstd. x is the normed input (s_out for the fused
 * add); ds (the gradient reaching the sum from its other use) may be NULL. */
int smelb_rmsnorm_bwd(const void* dy, const void* x, const void* w, int w_mode, const void* post_scale,
                      float post_mul, const float* rstd, const void* ds, int64_t rows, int64_t C, void* dx,
                      void* stream);

/* ---------------------------------------------------------------------------------------------------- experts
 * smel/moe.py:110-126 FrozenExpertsFn.forward / frozen_experts_forward: xs bf16 [rows, H] grouped by expert with
 * counts (device int32 [E], sum = rows); int4 bank gate_up (q [E, 2I, H/2], sz_t [E, H/64, 2I]) and down
 * (q [E, H, I/2], sz_t [E, I/64, H]); out bf16 [rows, H]. h_save (bf16 [rows, 2I]) may be NULL; a_buf
 * (bf16 [rows, I]) is caller scratch. The int4 unpack and group-64 dequant happen inside the GEMM producer. */
int smelb_frozen_experts_fwd(const void* xs, int64_t rows, int64_t H, int64_t I, const int32_t* counts, int64_t E,
                             const void* gu_q, const uint32_t* gu_sz, const void* dn_q, const uint32_t* dn_sz,
                             int act, void* h_save, void* a_buf, void* out, void* stream);

/* smel/moe.py:128-143 FrozenExpertsFn.backward: dx = dh @ W_gu with dh from dy @ W_dn and the activation gradient
 * (fp32). h (bf16 [rows, 2I]) is the saved gate/up pre-activation; when NULL it is recomputed into dh_buf's
 * companion h_buf. dh_buf bf16 [rows, 2I] and h_buf bf16 [rows, 2I] are caller scratch. */
int smelb_frozen_experts_bwd(const void* xs, const void* dy, int64_t rows, int64_t H, int64_t I,
                             const int32_t* counts, int64_t E, const void* gu_q, const uint32_t* gu_sz,
                             const void* dn_q, const uint32_t* dn_sz, int act, const void* h, void* h_buf,
                             void* dh_buf, void* dx, void* stream);

/* smel/moe.py:18-32 BF16Experts through FrozenExpertsFn (moe.py:110-143): the same two calls over a bf16 bank,
 * gate_up bf16 [E, 2I, H] and down bf16 [E, H, I], with the bank's tiles loaded by TMA instead of dequantized. */
int smelb_frozen_experts_bf16_fwd(const void* xs, int64_t rows, int64_t H, int64_t I, const int32_t* counts,
                                  int64_t E, const void* gate_up, const void* down, int act, void* h_save, void* a_buf,
                                  void* out, void* stream);
int smelb_frozen_experts_bf16_bwd(const void* xs, const void* dy, int64_t rows, int64_t H, int64_t I,
                                  const int32_t* counts, int64_t E, const void* gate_up, const void* down, int act,
                                  const void* h, void* h_buf, void* dh_buf, void* dx, void* stream);

/* ---------------------------------------------------------------------------------------------------- lora_linear
 * smel/lora.py:61-69 lora_linear and smel/lora.py:72-83 lora_gate_up: y bf16 [T, out] = x [T, in] w^T +
 * scale * (x A^T) B^T, computed as one GEMM whose last k-block is the LoRA term (the reference adds it in the addmm
 * epilogue before rounding as well). x, w (bf16 [out, in]) and y are bf16; A (fp32 [r, in]) and B (fp32 [out', r])
 * are the LoRA parameters. One pair (A0, B0; out' = out) is lora_linear; two pairs (A0, B0, A1, B1; out' = out / 2)
 * are lora_gate_up over the stacked [gate; up] weight, pair b acting on output rows [b out/2, (b+1) out/2). No pair
 * (A0 = B0 = NULL) is the plain x w^T. in and out are multiples of 64, r a multiple of 8 with (pairs * r) <= 64.
 * xa (bf16 [T, 64]) receives x [A0; A1]^T, which the backward reads; workspace: 256-byte aligned,
 * smelb_lora_linear_workspace_bytes(T, in, out) bytes. */
int64_t smelb_lora_linear_workspace_bytes(int64_t T, int64_t in_features, int64_t out_features);
int smelb_lora_linear_fwd(const void* x, int64_t T, int64_t in_features, const void* w, int64_t out_features,
                          const float* A0, const float* B0, const float* A1, const float* B1, int64_t r, float scale,
                          void* y, void* xa, void* workspace, int64_t workspace_bytes, void* stream);

/* Backward of smelb_lora_linear_fwd for dy (bf16 [T, out]): dx (bf16 [T, in]) = dy w + scale (dy B) A per pair,
 * gA_b (fp32, A_b's shape) = scale (dy_b B_b)^T x and gB_b (fp32, B_b's shape) = scale dy_b^T (x A_b^T), with dy_b
 * the pair's output columns. Any of dx / gA_b / gB_b may be NULL (not computed). xa is the forward's. */
int smelb_lora_linear_bwd(const void* x, const void* dy, int64_t T, int64_t in_features, const void* w,
                          int64_t out_features, const float* A0, const float* B0, const float* A1, const float* B1,
                          int64_t r, float scale, const void* xa, void* dx, float* gA0, float* gB0, float* gA1,
                          float* gB1, void* workspace, int64_t workspace_bytes, void* stream);

/* No counterpart in the reference. smelb_frozen_experts_fwd without caller scratch and without any allocation:
 * the activated intermediate (bf16 [rows, I]) lives in a file-scope device array of
 * SMELB_NOALLOC_SCRATCH_BYTES (plus a 256-byte head of wait-timeout status words), so rows * I * 2 may not exceed
 * SMELB_NOALLOC_SCRATCH_BYTES; larger calls return SMELB_ERR_SHAPE with the limit in smelb_last_error. The first
 * call on a device resolves the array's address (cudaGetSymbolAddress) with that device current; make that first
 * call before any stream capture. Every call on a device shares the array, so calls whose kernels overlap on the
 * GPU (different streams without ordering) race. Each call clears the status head first; a bounded wait that gives
 * up inside this call is recorded there, not in smelb_read_status: read it with
 * smelb_frozen_experts_fwd_noalloc_status. Same arguments as smelb_frozen_experts_fwd minus a_buf. */
#define SMELB_NOALLOC_SCRATCH_BYTES 33554432LL
int smelb_frozen_experts_fwd_noalloc(const void* xs, int64_t rows, int64_t H, int64_t I, const int32_t* counts,
                                     int64_t E, const void* gu_q, const uint32_t* gu_sz, const void* dn_q,
                                     const uint32_t* dn_sz, int act, void* h_save, void* out, void* stream);

/* No counterpart in the reference. The status head of smelb_frozen_experts_fwd_noalloc on `device`: synchronizes the
 * device and copies it out without allocating. words[0] is 0, or the code of a bounded device-side wait that gave up
 * during the last call (that call's output is then incomplete); words[1..3] the block, tile and k-block where it did.
 * reset != 0 clears the head. words has 4 entries. */
int smelb_frozen_experts_fwd_noalloc_status(int device, int* words, int reset);

/* ---------------------------------------------------------------------------------------------------- the layer
 * smel/moe.py:255-263 moe_forward (route -> routed_experts -> + shared_mlp) and its autograd backward, as two calls.
 * The flags select sub-paths so the same calls also serve route (moe.py:162-167), routed_experts (moe.py:214-252)
 * and mlp_lora / shared_mlp (moe.py:183-201). */
#define SMELB_F_ROUTER 1       /* compute routing from x and w_router (else topv_in / topi_in are used) */
#define SMELB_F_ROUTED 2       /* routed experts (frozen int4 bank + selected bf16 experts with LoRA) */
#define SMELB_F_SHARED 4       /* shared expert / dense MLP with LoRA */
#define SMELB_F_SHARED_GATE 8  /* multiply the shared expert by sigmoid(x @ w_sgate^T) */
#define SMELB_F_SAVE 16        /* keep activations for smelb_moe_layer_bwd */
#define SMELB_F_TOPV_FP32 32   /* topv / topv_in are fp32 (Gemma 4 routing) */
#define SMELB_F_RECOMPUTE 64   /* backward: h / sh_h were not kept by the forward; recompute them from x / xs first */
#define SMELB_F_EXT_DISPATCH 128 /* routed experts on a dispatch the caller built: xs, counts, gcounts, offsets, src_of,
                                  * row_of and total are inputs (max_rows dispatch rows), y (forward) and dxs
                                  * (backward) are the outputs in dispatch order; no router, gather, combine or dX
                                  * reduction run (the expert-parallel owner side). With SMELB_F_SHARED the shared
                                  * expert runs on the T rows of x in the same launches and leaves sh_y (and
                                  * sgate_logit; backward: sh_dx and dgl from g) to the caller. */

typedef struct smelb_moe_layer {
  /* shapes */
  int64_t T, H, E, K;   /* tokens, hidden, experts, top-k */
  int64_t I;            /* routed expert intermediate size */
  int64_t S;            /* shared expert intermediate size */
  int64_t n_sel;        /* selected (trainable bf16) experts */
  int64_t r_sel, r_sh;  /* LoRA ranks (0 = no LoRA) */
  float s_sel, s_sh;    /* LoRA scales alpha / r */
  int32_t act;          /* SMELB_ACT_* */
  int32_t flags;        /* SMELB_F_* */
  int64_t max_rows;     /* rows of the dispatch buffers: T*K + n_sel*64 */
  void* stream;
  /* inputs */
  const void* x;            /* bf16 [T, H] */
  const void* w_router;     /* bf16 [E, H] */
  const void* w_sgate;      /* bf16 [1, H] */
  const void* topv_in;      /* [T, K] when routing is given */
  const int64_t* topi_in;   /* [T, K] */
  const int32_t* tok_count; /* device int32 [1] = T */
  const void* gu_q; const uint32_t* gu_sz; /* [E, 2I, H/2] u8, [E, H/64, 2I] */
  const void* dn_q; const uint32_t* dn_sz; /* [E, H, I/2] u8, [E, I/64, H] */
  const int32_t* frozen_ids; /* device int32 [E - n_sel], ascending */
  const int32_t* sel_ids;    /* device int32 [n_sel], slot order */
  const int32_t* sel_slots;  /* device int32 [n_sel] = 0..n_sel-1 */
  const uint8_t* sel_mask;   /* device uint8 [E] */
  const void* sel_gu;        /* bf16 [n_sel, 2I, H] */
  const void* sel_dn;        /* bf16 [n_sel, H, I] */
  const float *A_gate, *B_gate, *A_up, *B_up, *A_down, *B_down; /* [n,r,H] [n,I,r] [n,r,H] [n,I,r] [n,r,I] [n,H,r] */
  const void* sh_gu;         /* bf16 [2S, H]: gate rows then up rows */
  const void* sh_dn;         /* bf16 [H, S] */
  const float *shA_gate, *shB_gate, *shA_up, *shB_up, *shA_down, *shB_down;
  /* outputs and activations (bf16 unless noted; R = max_rows; W64 = 64 columns, zero-initialised) */
  void* out;                /* [T, H] */
  float* probs;             /* fp32 [T, E] */
  void* topv;               /* [T, K] */
  int64_t* topi;            /* [T, K] */
  void* logits;             /* [T, E] */
  void* sgate_logit;        /* [T] */
  int32_t *counts, *gcounts, *offsets, *row_of, *src_of, *total; /* [E] [E] [E] [T*K] [R] [1] */
  int64_t* order;           /* [T*K] */
  void *xs, *h, *a, *y;     /* [R, H] [R, 2I] [R, I] [R, H] */
  void *xa, *z;             /* [R, W64] */
  void *sh_xa, *sh_h, *sh_a, *sh_z, *sh_y; /* [T, W64] [T, 2S] [T, S] [T, W64] [T, H] */
  void *p_xa_w, *p_gu_ext, *p_z_w, *p_dn_ext;     /* [n,2r,H] [n,2I,W64] [n,r,I] [n,H,W64] */
  void *sp_xa_w, *sp_gu_ext, *sp_z_w, *sp_dn_ext; /* [2r,H] [2S,W64] [r,S] [H,W64] */
  /* backward */
  const void* g;            /* [T, H] upstream gradient */
  void* dx;                 /* [T, H] */
  void *dy, *dh, *dxs;      /* [R, H] [R, 2I] [R, H] */
  void *dz, *dxa;           /* [R, W64] */
  void *dtopv, *dlogits, *dx_router; /* [T, K] [T, Epad64] zero-initialised, [T, H] */
  void *sh_dy, *sh_dh, *sh_dx;       /* [T, H] [T, 2S] [T, H] */
  void *sh_dz, *sh_dxa;              /* [T, W64] */
  float* dgl;                        /* fp32 [T] */
  void *p_dz_w, *p_da_ext, *p_dxa_w, *p_dx_ext;     /* [n,r,H] [n,I,W64] [n,2r,2I] [n,H,W64] */
  void *sp_dz_w, *sp_da_ext, *sp_dxa_w, *sp_dx_ext; /* [r,H] [S,W64] [2r,2S] [H,W64] */
  float *gA_gate, *gB_gate, *gA_up, *gB_up, *gA_down, *gB_down;             /* LoRA grads, shapes of the params */
  float *gshA_gate, *gshB_gate, *gshA_up, *gshB_up, *gshA_down, *gshB_down;
  /* optional */
  const float* dprobs;      /* fp32 [T, E] gradient w.r.t. probs (F_ROUTER backward), may be NULL */
  const void* fz_gu;        /* frozen bank in bf16 instead of int4 (gu_q == NULL): [E, 2I, H] (moe.py:18-32) */
  const void* fz_dn;        /* [E, H, I] */
  int32_t act_sh;           /* activation of the shared expert / dense MLP (SMELB_ACT_*) */
  int32_t reserved;
  const void* per_expert_scale; /* bf16 [E] multiplier of the renormalised top-k weights (Gemma 4), or NULL */
  int32_t* split_counts;    /* int32 [2 E] scratch of the small-token path: with at least 1024 dispatch rows on the
                               GEMV (smelb_set_gemv_rows), experts with more than 16 rows stay on the tile engine
                               and the rest take the GEMV; NULL: every frozen expert takes the GEMV */
} smelb_moe_layer;

/* ---------------------------------------------------------------------------------------------------- expert parallel
 * smel/moe.py:255-263 partitioned by expert over the P ranks (GPUs) of one box; the reference itself runs on one GPU,
 * so these entry points have no reference counterpart beyond the layer they partition. Each rank owns one region
 * (smelb_ep_region_alloc: cudaMalloc'd here, shared by CUDA IPC; smelb_ep_region_open maps a peer's) with four
 * exchange buffers of [P][cap][H] bf16 rows: 0 forward dispatch, 1 forward return, 2 backward dispatch, 3 backward
 * return. A sender writes into its own region and publishes; readers pull from the sender's region and acknowledge.
 * `regions` is a host array of the P region pointers as mapped in this process (regions[rank] its own); `cap` is
 * the most tokens a rank brings to one call. All synchronisation is on the device (smelb_ep_sync), with bounded
 * waits that record a status code; nothing synchronises with the host. */
#define SMELB_EP_WAIT_DONE 0  /* sender: every reader acknowledged the buffer's previous epoch */
#define SMELB_EP_PUBLISH 1    /* sender: publish the buffer's next epoch (its data is written) */
#define SMELB_EP_WAIT_READY 2 /* reader: every sender published the epoch this reader expects */
#define SMELB_EP_ACK 3        /* reader: done reading every sender's buffer of this epoch */
int64_t smelb_ep_region_bytes(int64_t P, int64_t cap, int64_t K, int64_t H);
int smelb_ep_region_alloc(int64_t bytes, void** region, void* ipc_handle /* 64 bytes out */);
int smelb_ep_region_open(const void* ipc_handle, void** region);
int smelb_ep_region_close(void* region);
int smelb_ep_region_free(void* region);
int smelb_ep_sync(const void* const* regions, int64_t P, int64_t rank, int64_t cap, int64_t K, int64_t H, int op,
                  int buffer, void* stream);

/* Source side, forward: per destination rank d the tokens with at least one expert that d owns (owner[E], local id
 * local_id[E]), in token order, de-duplicated (one row per token and destination), with their entries (local expert,
 * k, routing weight topv[t][k], bf16 or fp32) written into buffer 0's metadata. pos [T][P]: row of token t in d's
 * list or -1; slot_j [T][K]: slot of choice (t, k) within its row; tok_of [P][cap]: token of each row. T <= cap. */
int smelb_ep_plan(const int64_t* topi, const void* topv, int topv_fp32, int64_t T, int64_t K, const int32_t* owner,
                  const int32_t* local_id, const void* const* regions, int64_t P, int64_t rank, int64_t cap, int64_t H,
                  int32_t* pos, int32_t* slot_j, int32_t* tok_of, void* stream);

/* Source side: rows[buffer][d][i] = src[tok_of[d][i]] (buffer 0: token rows, 2: upstream gradient rows). */
int smelb_ep_pack_rows(const void* src, int64_t H, const int32_t* tok_of, const void* const* regions, int64_t P,
                       int64_t rank, int64_t cap, int64_t K, int buffer, void* stream);

/* Owner side: the dispatch entries every source sent (buffer 0), numbered in (source, row, slot) order: entry_e
 * (int64 [cap_entries], the local expert, `sink` past the received entries), entry_row (source row s * cap + i),
 * entry_w (routing weight); per source row its first entry and entry count (row_beg, row_m [P][cap]); rows received
 * per source (recv_rows [P]); n_total [1]. More than cap_entries entries record a status code. */
int smelb_ep_recv_plan(const void* const* regions, int64_t P, int64_t rank, int64_t cap, int64_t K, int64_t H,
                       int64_t cap_entries, int64_t sink, int64_t* entry_e, int32_t* entry_row, float* entry_w,
                       int32_t* row_beg, int32_t* row_m, int32_t* recv_rows, int32_t* n_total, void* stream);

/* Owner side: local [P][cap][H] = every source's rows of buffer 0 or 2 addressed to this rank (one NVLink pull per
 * row). */
int smelb_ep_pull_rows(const void* const* regions, int64_t P, int64_t rank, int64_t cap, int64_t K, int64_t H,
                       int buffer, void* local, void* stream);

/* Owner side: xs[row] = local[entry_row[src_of[row]]] for the dispatch rows before offsets[sink] (zeros on padding
 * rows), the dispatch plan being smelb_dispatch_plan_ws over entry_e with E = sink + 1. */
int smelb_ep_gather(const void* local, const int32_t* entry_row, const int32_t* src_of, const int32_t* offsets,
                    int64_t sink, int64_t H, int64_t max_rows, void* xs, void* stream);

/* Owner side: per received row, forward (backward = 0): sum over its entries of entry_w * y[row_of[entry]] (fp32,
 * slot order, rounded to bf16) into buffer 1; backward: the entries' dX rows y = dxs summed into buffer 3 and each
 * entry's d weight entry_dw into buffer 3's metadata. H % 256 == 0. */
int smelb_ep_return(const void* y, const int32_t* row_of, const float* entry_w, const float* entry_dw,
                    const int32_t* row_beg, const int32_t* row_m, const int32_t* recv_rows, const void* const* regions,
                    int64_t P, int64_t rank, int64_t cap, int64_t K, int64_t H, int backward, void* stream);

/* Owner side, backward: dy[row] = bf16(g * w) of each dispatch row's entry (g: the pulled gradient rows, local) and
 * entry_dw[entry] = sum_h g[h] * y[row][h] in fp32 (y: the forward's expert outputs in dispatch order). */
int smelb_ep_dy(const void* g_local, const int32_t* entry_row, const float* entry_w, const int32_t* src_of,
                const int32_t* offsets, int64_t sink, int64_t H, int64_t max_rows, const void* y, void* dy,
                float* entry_dw, void* stream);

/* Source side: out[t] = bf16(a[t] + the returned rows (buffer 1, or 3 when backward) at pos[t][d] over the
 * destinations in rank order, in fp32), where a = add (bf16 [T, H]; zero when add is NULL), gated in the forward by
 * the shared expert's gate when gate_logit (bf16 [T]) is given: a = bf16(add * bf16(sigmoid(gate_logit))), the fused
 * layer's combine (smel/moe.py:197-201,248-252). Backward: + dgl[t] * w_sgate (fp32 [T], bf16 [H]; the shared gate's
 * share of dX, when given), and dtopv[t][k] (bf16, or fp32 if dtopv_fp32) from the owners' per-entry d weights. */
int smelb_ep_collect(const void* const* regions, int64_t P, int64_t rank, int64_t cap, int64_t K, int64_t H, int64_t T,
                     const int32_t* pos, const void* add, const void* gate_logit, const float* dgl,
                     const void* w_sgate, int backward, const int64_t* topi, const int32_t* owner,
                     const int32_t* slot_j, void* dtopv, int dtopv_fp32, void* out, void* stream);

/* ---------------------------------------------------------------------------------------------------- int8 rows
 * smel/quant.py:97-105 quantize_int8_rows / dequant_int8_rows: symmetric int8 per row of w (bf16, or fp32 when
 * w_fp32) [rows, H]: s = max(amax|w| / 127, 1e-12) (fp32), q = clamp(round_half_even(w / s), -127, 127) (int8
 * [rows, H]), scale = bf16(s) [rows]; dequant: out [rows, H] = q * scale rounded once to bf16, or fp32 when
 * out_fp32. */
int smelb_int8_rows_quantize(const void* w, int w_fp32, int64_t rows, int64_t H, void* q, void* scale, void* stream);
int smelb_int8_rows_dequant(const void* q, const void* scale, int64_t rows, int64_t H, void* out, int out_fp32,
                            void* stream);

/* ---------------------------------------------------------------------------------------------------- chunked CE
 * smel/loss.py:130-156 chunked_ce / _ChunkedCE.forward, each token chunk one pass of smel/loss.py:50-92 _ce_chunk
 * over the vocabulary chunks: the cross-entropy of the hidden rows h (bf16 [N, H], H % 64 == 0) against tgt
 * (int64 [N]) over a frozen LM head, the gradient accumulated online under the log-sum-exp's running maximum.
 * Head: bf16 rows w [V, H], or int8 rows q [V, H] with a bf16 scale per row q_scale [V] (smel/quant.py:97-105);
 * pass exactly one of the two. softcap > 0 caps the logits as cap * tanh(z / cap) (smel/loss.py:34-35), gradient
 * included. Outputs: loss_rows (fp32 [N]) = lse - target logit per row (a target outside [0, V) contributes lse);
 * loss (fp32 [1]) = sum(loss_rows) / denom; gh (bf16 [N, H]) = d loss / d h, or NULL for the loss alone.
 * workspace: 256-byte aligned, smelb_chunked_ce_workspace_bytes(N, token_chunk, H, min(V, vocab_chunk), int8,
 * gh != NULL) bytes. The vocabulary chunks are the outer loop (an int8 head is dequantised once per call), so the
 * online state of all N rows lives in the workspace; token_chunk bounds the [token_chunk, vocab_chunk] logit tile. */
int64_t smelb_chunked_ce_workspace_bytes(int64_t N, int64_t token_chunk, int64_t H, int64_t vocab_chunk, int int8,
                                         int need_grad);
int smelb_chunked_ce(const void* h, const int64_t* tgt, int64_t N, int64_t H, const void* w, const void* q,
                     const void* q_scale, int64_t V, int64_t vocab_chunk, int64_t token_chunk, float softcap,
                     float denom, float* loss_rows, float* loss, void* gh, void* workspace, int64_t workspace_bytes,
                     void* stream);

/* smel/loss.py:45-47 LMHead.logits: out (fp32 [N, V]) = cap(float(bf16(h @ W^T))) chunk by chunk over the
 * vocabulary; the head as for smelb_chunked_ce. workspace: 256-byte aligned,
 * smelb_lm_logits_workspace_bytes(N, H, min(V, vocab_chunk), int8) bytes. */
int64_t smelb_lm_logits_workspace_bytes(int64_t N, int64_t H, int64_t vocab_chunk, int int8);
int smelb_lm_logits(const void* h, int64_t N, int64_t H, const void* w, const void* q, const void* q_scale, int64_t V,
                    int64_t vocab_chunk, float softcap, float* out, void* workspace, int64_t workspace_bytes,
                    void* stream);

/* Instrumentation. smelb_launch_count: kernels launched by this library so far (all entry points).
 * smelb_gemm_timing(1) records a CUDA event pair on the launching stream around every expert-GEMM launch;
 * smelb_gemm_timing_read synchronizes on them and returns the summed duration (ms) and the number of launches
 * recorded since the previous read. */
long long smelb_launch_count(void);
int smelb_gemm_timing(int enable);
/* Dispatch-row count at or below which the forward's frozen int4 experts (smelb_moe_layer_fwd, and
 * smelb_frozen_experts_fwd over its rows) run as a dequant-GEMV instead of the tile engine; returns the previous
 * value (default 512; 0 keeps every call on the tile engine). Within it, layer calls of at most 6 tokens also take
 * the router / shared-gate logits and the shared expert (without its LoRA) as dense GEMVs. Replaces the size switch
 * of no reference interface: smel/moe.py:58-85 has one path at every size. */
int64_t smelb_set_gemv_rows(int64_t rows);
int smelb_gemm_timing_read(double* ms_total, long long* launches);

/* sizeof(smelb_moe_layer), for bindings to check their mirror of the struct. */
size_t smelb_moe_layer_size(void);

int smelb_moe_layer_fwd(const smelb_moe_layer* L);
int smelb_moe_layer_bwd(const smelb_moe_layer* L);

#ifdef __cplusplus
}
#endif

#endif /* SMELB_H */
