// Host entry points of the memory-bound MoE kernels (kernels.cu). All return a Status code.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

namespace smelb {

using bf16 = __nv_bfloat16;

struct PackBlock {
  const float* src;  // nullptr: block unused
  long long sj;      // source stride between slots j
  long long sa, sb;  // source strides along the output's a / b axes
  int a0, na, b0, nb;
  float scale;
};
struct PackSpec {
  int J, OA, OB;
  PackBlock blk[2];
};
// Several pack outputs in one launch (the LoRA operands of one layer call).
constexpr int kMaxPacks = 8;
struct PackBatch {
  int n;
  PackSpec spec[kMaxPacks];
  void* out[kMaxPacks];
  long long start[kMaxPacks + 1];  // prefix of the output element counts
  int rstart[kMaxPacks + 1];       // prefix of the output rows (J * OA)
};

// stepwise: bf16 output rounded after the product and again after the sum (torch's bf16 ops, smel/quant.py:87-94)
int int4_dequant(const void* q, const void* scale, const void* zero, void* out, long long rows, int k, int groups,
                 bool out_f32, cudaStream_t st, bool stepwise = false);
// out = w + fl(scale * B) @ A (fp32 fma chain over the rank, one rounding to w's dtype): w, out [rows, cols] bf16
// (fp32 when f32), B fp32 [rows, r], A fp32 [r, cols]. out may equal w.
int lora_merge(const void* w, bool f32, const float* B, const float* A, int rows, int cols, int r, float scale,
               void* out, cudaStream_t st);
// Group-64 int4 quantizer with the clip search of smel/quant.py:5-44 (up to kMaxClip candidate factors).
constexpr int kMaxClip = 8;
int int4_quantize(const void* w, bool w_f32, long long rows, int k, const float* clip, int n_clip, void* q,
                  void* scale, void* zero, cudaStream_t st);
int int4_pack_sz(const void* scale, const void* zero, uint32_t* szT, long long nw, int rows, int groups,
                 cudaStream_t st);
int router_topk(const void* logits, long long ld, int T, int E, int K, float* probs, void* topv, bool topv_f32,
                long long* topi, const void* per_expert_scale, cudaStream_t st);
int router_bwd(const void* dtopv, bool dtopv_f32, const float* dprobs, const float* probs, const long long* topi,
               const void* per_expert_scale, int T, int E, int K, void* dlogits, long long ld, cudaStream_t st);
int dispatch_plan(const long long* topi, long long R, int E, const uint8_t* sel_mask, int pad, int* counts,
                  int* gcounts, int* offsets, int* row_of, int* src_of, long long* order, int* total, cudaStream_t st);
// The same plan on many CTAs, with `scratch` (>= 2 * E ints useful; nb x E used) lent by the caller.
int dispatch_plan_mt(const long long* topi, long long R, int E, const uint8_t* sel_mask, int pad, int* counts,
                     int* gcounts, int* offsets, int* row_of, int* src_of, long long* order, int* total, int* scratch,
                     long long scratch_ints, cudaStream_t st);
int gather_rows(const void* x, int H, int K, const int* src_of, const int* total, long long max_rows, void* xs,
                cudaStream_t st);
int combine_fwd(const void* y, const int* row_of, const void* topv, bool topv_f32, int T, int K, int H,
                const void* y_sh, const void* gl, void* out, cudaStream_t st);
int combine_bwd_rows(const void* g, const void* y, const int* src_of, const int* total, long long max_rows,
                     const void* topv, bool topv_f32, int K, int H, void* dy, void* dtopv, cudaStream_t st);
int shared_gate_bwd(const void* g, const void* y_sh, const void* gl, int T, int H, void* dy_sh, float* dgl,
                    cudaStream_t st);
int dx_reduce(const void* dxs, const int* row_of, int K, int T, int H, const void* dx_sh, const void* dx_r,
              const float* dgl, const void* w_sg, void* dx, cudaStream_t st);
int pack_blocks(const PackSpec& spec, void* out, cudaStream_t st);
int pack_batch(PackBatch& batch, cudaStream_t st);  // launches nothing when the batch is empty

struct NormArgs {
  const bf16* x;
  const bf16* h;           // residual input of the fused add, or null
  const bf16* w;           // norm weight, or null (w_mode 0)
  const bf16* post_scale;  // router prologue scale vector, or null
  float post_mul;          // router prologue scalar (0: none)
  int w_mode;
  float eps;
  long long rows;
  int C;
  bf16* s;                 // fused add output (h + x), with h
  bf16* y;
  float* rstd;             // per-row rstd, or null
};

struct NormBwdArgs {
  const bf16* dy;
  const bf16* x;           // the normed input (the fused add's sum s for add_rmsnorm)
  const bf16* w;
  const bf16* post_scale;
  float post_mul;
  int w_mode;
  const float* rstd;
  const bf16* ds;          // gradient reaching the sum from its other use, or null
  long long rows;
  int C;
  bf16* dx;
};

// Chunked cross-entropy over a frozen LM head (smel/loss.py:50-92), the per-row steps around the two GEMMs of a
// vocabulary chunk. State per row: running max m, running sum s, the last rescale factor r, the target's (capped)
// logit, the cap's derivative at the target, the fp32 gradient accumulator [n, H] and the target's head row.
struct CeState {
  float *m, *s, *r, *tlog, *tdrv;
  float *acc, *tgt_row;  // [n, H]
};
int ce_init(const CeState& st, long long n, int H, cudaStream_t s);
// p[i] = min(step, total - i * step), i < nchunks (the device-side token counts of the GEMMs, one per chunk)
int set_counts(int* p, int nchunks, int step, long long total, cudaStream_t s);
// lg: bf16 logits [n, ld] of the chunk's Vc columns (vocabulary rows v0 .. v0 + Vc - 1), overwritten in place by p,
// the softmax numerators times the cap's derivative (bf16, zero in columns Vc .. ld - 1) when need_grad.
int ce_rows(void* lg, int ld, int Vc, long long v0, const long long* tgt, float softcap, bool need_grad,
            const void* wc, int H, const CeState& st, long long n, cudaStream_t s);
// acc = acc * r + sum of the nparts fp32 partial products [nparts][n, H] (the chunk's p @ W, split along the chunk)
int ce_acc(const float* parts, int nparts, const CeState& st, long long n, int H, cudaStream_t s);
// loss_rows = m + log s - tlog; gh (bf16, may be NULL) = (acc / s - tdrv * tgt_row) / denom
int ce_finish(const CeState& st, long long n, int H, float denom, float* loss_rows, void* gh, cudaStream_t s);
// out[row, v] (fp32, row pitch ldo) = cap(float(lg[row, v])) for the chunk's Vc columns
int ce_logits_out(const void* lg, int ld, int Vc, long long n, float softcap, float* out, long long ldo,
                  cudaStream_t s);
// loss = sum(loss_rows) / denom (one block, fixed order)
int ce_loss_sum(const float* loss_rows, long long n, float denom, float* loss, cudaStream_t s);
// w (bf16 or fp32 [rows, H]) -> int8 rows q [rows, H] + bf16 scale [rows] (smel/quant.py:97-101)
int int8_rows_quantize(const void* w, bool w_fp32, long long rows, int H, void* q, void* scale, cudaStream_t s);
// int8 rows (symmetric, bf16 scale per row) -> bf16 or fp32: q * scale rounded once (smel/quant.py:104-105)
int int8_rows_dequant(const void* q, const void* scale, long long rows, int H, void* out, cudaStream_t s,
                      bool out_fp32 = false);

// Small-token dequant-GEMV over a frozen int4 bank (gemv.cu): the rows of expert ids[i] (i itself when ids is null)
// are the token rows offsets[e] .. offsets[e] + counts[e] - 1 of xs (without offsets: the experts' rows follow one
// another in id order); q [E][rows_w][K/2], sz [E][K/64][rows_w] (scale | zero << 16).
// glu: out[., inter] = act(x W[0:inter]^T) * (x W[inter:2 inter]^T), pre-activations into hout when given;
// otherwise out[., rows_w] = x W^T. tok_hint: the expected rows per active expert (sizes the token tile).
struct GemvArgs {
  const bf16* xs;
  long long ldx;
  const int *counts, *offsets, *ids;
  int n_ids;
  int n_experts;  // experts in the bank (bounds of q / sz)
  const uint8_t* q;
  const uint32_t* sz;
  int rows_w, K, inter, act;
  bool glu;
  int tok_hint;
  bf16* out;
  long long ldo;
  bf16* hout;
  long long ldh;
};
int int4_gemv(const GemvArgs& a, cudaStream_t st);
// hot[e] = counts[e] if counts[e] > thr else 0, cold[e] = the rest (e < E): the experts the tile engine and the GEMV
// take in a split small-token call.
int split_counts(const int* counts, int E, int thr, int* hot, int* cold, cudaStream_t st);
// Whether the GEMV takes a reduction length K (its shared-memory stages must hold two tasks).
bool int4_gemv_supported(bool glu, int K);

// Small-token dense projection with bf16 weights (the shared expert at a handful of tokens):
// out[t][m] = bf16(sum_k W[m][k] x[t][k]) for m < M, or with glu, over the gate row f and the up row inter + f,
// g = bf16(.), u = bf16(.), out[t][f] = bf16(bf16(act(g)) * u) for f < inter, (g | u) into hout when given.
struct DenseGemvArgs {
  const bf16* w;  // [M][ldw], M = 2 * inter with glu
  long long ldw;
  int M;
  const bf16* x;  // [T][ldx]
  long long ldx;
  int T, K;
  bool glu;
  int inter, act;
  bf16* out;
  long long ldo;
  bf16* hout;
  long long ldh;
  // optional second plain projection of the same tokens in the same launch (units M .. M + M2 - 1): out2[t][m] =
  // bf16(sum_k W2[m][k] x[t][k]); not with glu
  const bf16* w2;
  long long ldw2;
  int M2;
  bf16* out2;
  long long ldo2;
};
// Its FMA work grows with the tokens (~3 us per token for the Qwen3.6 shared expert against ~0.5 us for the engine's
// tiles; 7.3 against 23.7 us at one token, 52 against 32 at sixteen), so it takes up to 6 tokens.
constexpr int kDenseGemvMaxT = 6;
// Whether dense_gemv takes these sizes and pointers (T <= kDenseGemvMaxT, K a multiple of 8 up to 4096, 16-byte
// aligned rows); callers take the GEMM engine otherwise.
bool dense_gemv_supported(const DenseGemvArgs& a);
int dense_gemv(const DenseGemvArgs& a, cudaStream_t st);

int rmsnorm_fwd(const NormArgs& a, cudaStream_t st);
int rmsnorm_bwd(const NormBwdArgs& a, cudaStream_t st);

int launch_gemm(struct LaunchArgs& args, cudaStream_t stream);
// Same launch with the wait-timeout status words supplied by the caller (4 ints, device memory) instead of the
// per-device word launch_gemm allocates on first use (timing and launch count as launch_gemm).
int launch_gemm_status(struct LaunchArgs& args, cudaStream_t stream, int* err);

}  // namespace smelb
