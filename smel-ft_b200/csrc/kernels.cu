// Memory-bound kernels of the MoE layer: int4 dequant (parity helper) and (scale, zero) repack, router softmax /
// top-k / renorm and its backward, the deterministic counting-sort dispatch, row gather, the fp32 weighted combine
// and its backward, the final dX reduction and the per-step LoRA factor packing.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "host.h"

namespace smelb {

// ============================================================================================ int4 dequant
// out[r][2j] = lo(q[r][j]) * s + z, out[r][2j+1] = hi(q[r][j]) * s + z with (s, z) of group (2j) / group_size.
// Single (smel/quant.py:51-67, the Triton kernel): computed in fp32 and rounded once to the output type.
// Stepwise (smel/quant.py:87-94, dequant_int4_torch with a bf16 output): every operation in the output dtype, so the
// product q * s is rounded to bf16 before z is added and the sum is rounded again (q * s is exact in fp32, so this is
// torch's bf16 mul then bf16 add bit for bit). With an fp32 output the two modes are the same.
template <bool F32, bool kStepwise>
__global__ void int4_dequant_kernel(const uint8_t* __restrict__ q, const bf16* __restrict__ scale,
                                    const bf16* __restrict__ zero, void* __restrict__ out, long long rows, int half_k,
                                    int groups, int group) {
  const long long n = rows * half_k;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / half_k;
    const int j = (int)(i - r * half_k);
    const int g = (2 * j) / group;
    const float s = __bfloat162float(scale[r * groups + g]);
    const float z = __bfloat162float(zero[r * groups + g]);
    const uint8_t b = q[i];
    float lo, hi;
    if (kStepwise && !F32) {
      lo = bf16_round(bf16_round((float)(b & 0xF) * s) + z);
      hi = bf16_round(bf16_round((float)(b >> 4) * s) + z);
    } else {
      lo = fmaf((float)(b & 0xF), s, z);
      hi = fmaf((float)(b >> 4), s, z);
    }
    if (F32) {
      float2 v = make_float2(lo, hi);
      reinterpret_cast<float2*>(out)[i] = v;
    } else {
      reinterpret_cast<__nv_bfloat162*>(out)[i] = __floats2bfloat162_rn(lo, hi);
    }
  }
}

int int4_dequant(const void* q, const void* scale, const void* zero, void* out, long long rows, int k, int groups,
                 bool out_f32, cudaStream_t st, bool stepwise) {
  SMELB_CHECK_ARG(k > 0 && k % 2 == 0 && groups > 0 && k % groups == 0 && (k / groups) % 2 == 0, kErrShape,
                  "int4_dequant: k=%d groups=%d (need k %% groups == 0 and an even group size)", k, groups);
  if (rows == 0) return kOk;
  const long long n = rows * (k / 2);
  const int threads = 256;
  const long long blocks = std::min<long long>((n + threads - 1) / threads, 148LL * 16);
  const uint8_t* qb = (const uint8_t*)q;
  const bf16 *sb = (const bf16*)scale, *zb = (const bf16*)zero;
  if (out_f32)
    int4_dequant_kernel<true, false><<<(int)blocks, threads, 0, st>>>(qb, sb, zb, out, rows, k / 2, groups, k / groups);
  else if (stepwise)
    int4_dequant_kernel<false, true><<<(int)blocks, threads, 0, st>>>(qb, sb, zb, out, rows, k / 2, groups, k / groups);
  else
    int4_dequant_kernel<false, false><<<(int)blocks, threads, 0, st>>>(qb, sb, zb, out, rows, k / 2, groups, k / groups);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

// ============================================================================================ LoRA merge
// out[i][c] = round(w[i][c] + sum_k fl(scale * B[i][k]) * A[k][c]) (smel/pack.py merge_experts / merge_mlp with
// smel/lora.py delta()): the low-rank delta in fp32 as one fused multiply-add chain over k = 0..r-1 starting from 0
// (the order of the reference's fp32 matmul for this shape), added to the weight in fp32 and rounded once to the
// weight's dtype. One thread per output element; A's row k is shared by the block's threads through L1.
template <bool F32>
__global__ void lora_merge_kernel(const void* __restrict__ w, const float* __restrict__ B, const float* __restrict__ A,
                                  int rows, int cols, int r, float scale, void* __restrict__ out) {
  const long long n = (long long)rows * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int row = (int)(i / cols), c = (int)(i - (long long)row * cols);
    const float* b = B + (long long)row * r;
    float acc = 0.f;
    for (int k = 0; k < r; ++k) acc = fmaf(scale * __ldg(b + k), __ldg(A + (long long)k * cols + c), acc);
    if (F32) {
      reinterpret_cast<float*>(out)[i] = __fadd_rn(reinterpret_cast<const float*>(w)[i], acc);
    } else {
      const float wv = __bfloat162float(reinterpret_cast<const bf16*>(w)[i]);
      reinterpret_cast<bf16*>(out)[i] = __float2bfloat16_rn(__fadd_rn(wv, acc));
    }
  }
}

int lora_merge(const void* w, bool f32, const float* B, const float* A, int rows, int cols, int r, float scale,
               void* out, cudaStream_t st) {
  SMELB_CHECK_ARG(rows >= 0 && cols >= 0 && r >= 0, kErrShape, "lora_merge: rows=%d cols=%d r=%d", rows, cols, r);
  const long long n = (long long)rows * cols;
  if (n == 0) return kOk;
  const int threads = 256;
  const long long blocks = std::min<long long>((n + threads - 1) / threads, 148LL * 16);
  if (f32)
    lora_merge_kernel<true><<<(int)blocks, threads, 0, st>>>(w, B, A, rows, cols, r, scale, out);
  else
    lora_merge_kernel<false><<<(int)blocks, threads, 0, st>>>(w, B, A, rows, cols, r, scale, out);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

// ------------------------------------------------------------------------------------------ int4 quantizer
// smel/quant.py:5-44, one warp per 64-value group (lane l holds columns 2l, 2l+1, so the warp reads the group's
// 128 or 256 contiguous bytes and writes its 32 packed bytes). Every fp32 step is a separate correctly rounded
// operation in the reference's order (no contraction into FMAs): the group's [min, max], its center, each clip
// candidate's range, step = max((hi - lo) / 15, 1e-8) and base = lo both rounded to bf16, codes
// round_half_even((w - base) / step) clamped to [0, 15], and the squared error of codes * step + base. A later
// candidate replaces the best one only when its error is strictly smaller. The error sum runs as a butterfly over
// the warp, so where two candidates' errors agree to within fp32 rounding the choice can differ from the
// reference's CPU sum order.
struct ClipList {
  int n;
  float c[kMaxClip];
};

__device__ __forceinline__ float warp_sum_rn(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

template <bool F32>
__global__ void int4_quantize_kernel(const void* __restrict__ w, uint8_t* __restrict__ q, uint16_t* __restrict__ scale,
                                     uint16_t* __restrict__ zero, long long ngroups, ClipList cl) {
  const int lane = threadIdx.x & 31;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long gi = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; gi < ngroups; gi += nwarps) {
    float w0, w1;
    if (F32) {
      const float2 v = reinterpret_cast<const float2*>(w)[gi * 32 + lane];
      w0 = v.x;
      w1 = v.y;
    } else {
      const __nv_bfloat162 v = reinterpret_cast<const __nv_bfloat162*>(w)[gi * 32 + lane];
      w0 = __low2float(v);
      w1 = __high2float(v);
    }
    float mn = fminf(w0, w1), mx = fmaxf(w0, w1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const float mid = __fdiv_rn(__fadd_rn(mn, mx), 2.0f);
    float best_err = 0.0f, best_s = 0.0f, best_z = 0.0f, best_q0 = 0.0f, best_q1 = 0.0f;
    for (int ci = 0; ci < cl.n; ++ci) {
      const float c = cl.c[ci];
      const float lo = __fadd_rn(mid, __fmul_rn(__fsub_rn(mn, mid), c));
      const float hi = __fadd_rn(mid, __fmul_rn(__fsub_rn(mx, mid), c));
      const float s = __bfloat162float(__float2bfloat16_rn(fmaxf(__fdiv_rn(__fsub_rn(hi, lo), 15.0f), 1e-8f)));
      const float z = __bfloat162float(__float2bfloat16_rn(lo));
      const float q0 = fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(w0, z), s)), 0.0f), 15.0f);
      const float q1 = fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(w1, z), s)), 0.0f), 15.0f);
      const float d0 = __fsub_rn(__fadd_rn(__fmul_rn(q0, s), z), w0);
      const float d1 = __fsub_rn(__fadd_rn(__fmul_rn(q1, s), z), w1);
      const float e = warp_sum_rn(__fadd_rn(__fmul_rn(d0, d0), __fmul_rn(d1, d1)));
      if (ci == 0 || e < best_err) {
        best_err = e;
        best_s = s;
        best_z = z;
        best_q0 = q0;
        best_q1 = q1;
      }
    }
    q[gi * 32 + lane] = (uint8_t)((int)best_q0 | ((int)best_q1 << 4));
    if (lane == 0) {
      scale[gi] = __bfloat16_as_ushort(__float2bfloat16_rn(best_s));
      zero[gi] = __bfloat16_as_ushort(__float2bfloat16_rn(best_z));
    }
  }
}

int int4_quantize(const void* w, bool w_f32, long long rows, int k, const float* clip, int n_clip, void* q,
                  void* scale, void* zero, cudaStream_t st) {
  SMELB_CHECK_ARG(k > 0 && k % 64 == 0, kErrShape, "int4_quantize: k=%d is not a multiple of the group size 64", k);
  SMELB_CHECK_ARG(n_clip >= 1 && n_clip <= kMaxClip, kErrArg, "int4_quantize: %d clip factors (1..%d)", n_clip,
                  kMaxClip);
  SMELB_CHECK_ARG(rows >= 0, kErrShape, "int4_quantize: rows=%lld", rows);
  if (rows == 0) return kOk;
  ClipList cl;
  cl.n = n_clip;
  for (int i = 0; i < kMaxClip; ++i) cl.c[i] = i < n_clip ? clip[i] : 1.0f;
  const long long ngroups = rows * (k / 64);
  const int threads = 256;
  const long long blocks = std::min<long long>((ngroups + 7) / 8, 148LL * 16);
  if (w_f32)
    int4_quantize_kernel<true><<<(int)blocks, threads, 0, st>>>(w, (uint8_t*)q, (uint16_t*)scale, (uint16_t*)zero,
                                                                 ngroups, cl);
  else
    int4_quantize_kernel<false><<<(int)blocks, threads, 0, st>>>(w, (uint8_t*)q, (uint16_t*)scale, (uint16_t*)zero,
                                                                  ngroups, cl);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

// szT[w][g][r] = scale[w][r][g] | zero[w][r][g] << 16 : the (scale, zero) pairs of one group for consecutive rows are
// contiguous, which is the order the GEMM producer stages them in.
__global__ void int4_pack_sz_kernel(const uint16_t* __restrict__ scale, const uint16_t* __restrict__ zero,
                                    uint32_t* __restrict__ szT, long long nw, int rows, int groups) {
  const long long n = nw * rows * groups;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long w = i / ((long long)rows * groups);
    const long long rem = i - w * rows * groups;
    const int g = (int)(rem / rows), r = (int)(rem - (long long)g * rows);
    const long long src = (w * rows + r) * groups + g;
    szT[i] = (uint32_t)scale[src] | ((uint32_t)zero[src] << 16);
  }
}

int int4_pack_sz(const void* scale, const void* zero, uint32_t* szT, long long nw, int rows, int groups,
                 cudaStream_t st) {
  const long long n = nw * rows * groups;
  if (n == 0) return kOk;
  const long long blocks = std::min<long long>((n + 255) / 256, 148LL * 16);
  int4_pack_sz_kernel<<<(int)blocks, 256, 0, st>>>((const uint16_t*)scale, (const uint16_t*)zero, szT, nw, rows,
                                                   groups);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

// ============================================================================================ router
// One warp per token: probs = softmax_fp32(logits), top-k by (value desc, expert id asc), renormalised in fp32 over
// the chosen k (summed in k order), optionally multiplied by per_expert_scale (Gemma 4), stored as bf16 or fp32.
// Lane l holds experts l, l + 32, ..., kMaxPer of them (E <= 32 * kMaxPer): the top-k rounds scan only the slots an
// expert count can fill (the rounds are the kernel's time; a fixed 16 slots doubled it at 256 experts).
template <int kMaxPer>
__global__ void router_topk_kernel(const bf16* __restrict__ logits, long long ld, int T, int E, int K,
                                   float* __restrict__ probs, void* __restrict__ topv, int topv_f32,
                                   long long* __restrict__ topi, const bf16* __restrict__ per_expert_scale) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T) return;
  const bf16* lg = logits + (long long)warp * ld;
  float v[kMaxPer];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int e = lane + 32 * i;
    v[i] = (e < E) ? __bfloat162float(lg[e]) : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int e = lane + 32 * i;
    v[i] = (e < E) ? expf(v[i] - mx) : 0.f;
    sum += v[i];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv = 1.0f / sum;
  float* pr = probs + (long long)warp * E;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int e = lane + 32 * i;
    if (e < E) {
      v[i] = v[i] * inv;
      pr[e] = v[i];
    } else {
      v[i] = -INFINITY;
    }
  }
  // top-k: repeated warp arg-max; ties resolved towards the smaller expert id. Lane k keeps the k-th choice
  // (K <= 32), so the choices stay in registers.
  float myv = 0.f;
  int mye = 0;
  for (int k = 0; k < K; ++k) {
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      const int e = lane + 32 * i;
      if (v[i] > bv || (v[i] == bv && e < be)) {
        bv = v[i];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i)
      if (lane + 32 * i == be) v[i] = -INFINITY;
    if (lane == k) {
      myv = bv;
      mye = be;
    }
  }
  // the renormalising sum in k order (every lane forms the same sum), then lane k writes choice k
  float s = 0.f;
  for (int k = 0; k < K; ++k) s += __shfl_sync(0xffffffffu, myv, k);
  if (lane < K) {
    float val = myv / s;
    if (per_expert_scale) val = val * __bfloat162float(per_expert_scale[mye]);
    const long long o = (long long)warp * K + lane;
    if (topv_f32) reinterpret_cast<float*>(topv)[o] = val;
    else reinterpret_cast<bf16*>(topv)[o] = __float2bfloat16_rn(val);
    topi[o] = mye;
  }
}

int router_topk(const void* logits, long long ld, int T, int E, int K, float* probs, void* topv, bool topv_f32,
                long long* topi, const void* per_expert_scale, cudaStream_t st) {
  SMELB_CHECK_ARG(E >= 1 && E <= 512 && K >= 1 && K <= 32 && K <= E, kErrShape, "router_topk: E=%d K=%d", E, K);
  if (T == 0) return kOk;
  const int threads = 256;
  const int blocks = (T * 32 + threads - 1) / threads;
  auto kern = E <= 128 ? router_topk_kernel<4> : E <= 256 ? router_topk_kernel<8> : router_topk_kernel<16>;
  kern<<<blocks, threads, 0, st>>>((const bf16*)logits, ld, T, E, K, probs, topv, topv_f32 ? 1 : 0, topi,
                                   (const bf16*)per_expert_scale);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

// Backward of probs -> top-k gather -> renorm (-> optional per-expert scale) -> cast:
//   t_k = v_k / S, S = sum_j v_j;  dv_k = (dt_k - sum_j dt_j t_j) / S;  dp[e] = dprobs[e] + sum_k [topi_k == e] dv_k;
//   dl = p * (dp - sum_e dp_e p_e)  (softmax Jacobian), stored in the logits dtype (bf16). dprobs may be null.
__global__ void router_bwd_kernel(const void* __restrict__ dtopv, int dtopv_f32, const float* __restrict__ dprobs,
                                  const float* __restrict__ probs, const long long* __restrict__ topi,
                                  const bf16* __restrict__ per_expert_scale, int T, int E, int K,
                                  bf16* __restrict__ dlogits, long long ld) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T) return;
  const float* pr = probs + (long long)warp * E;
  const float* dpr = dprobs ? dprobs + (long long)warp * E : nullptr;
  float dv = 0.f;
  int myk_e = -1;
  if (lane < K) {
    float S = 0.f, dot = 0.f;
    for (int k = 0; k < K; ++k) S += pr[topi[(long long)warp * K + k]];
    for (int k = 0; k < K; ++k) {
      const long long o = (long long)warp * K + k;
      const int e = (int)topi[o];
      float d = dtopv ? (dtopv_f32 ? reinterpret_cast<const float*>(dtopv)[o]
                                   : __bfloat162float(reinterpret_cast<const bf16*>(dtopv)[o]))
                      : 0.f;
      if (per_expert_scale) d *= __bfloat162float(per_expert_scale[e]);
      dot += d * (pr[e] / S);
    }
    const long long o = (long long)warp * K + lane;
    myk_e = (int)topi[o];
    float d = dtopv ? (dtopv_f32 ? reinterpret_cast<const float*>(dtopv)[o]
                                 : __bfloat162float(reinterpret_cast<const bf16*>(dtopv)[o]))
                    : 0.f;
    if (per_expert_scale) d *= __bfloat162float(per_expert_scale[myk_e]);
    dv = (d - dot) / S;
  }
  // sdot = sum_e dp_e p_e
  float contrib = (lane < K) ? dv * pr[myk_e] : 0.f;
  if (dpr)
    for (int e = lane; e < E; e += 32) contrib += dpr[e] * pr[e];
#pragma unroll
  for (int o = 16; o; o >>= 1) contrib += __shfl_xor_sync(0xffffffffu, contrib, o);
  const float sdot = contrib;
  bf16* dl = dlogits + (long long)warp * ld;
  for (int e0 = 0; e0 < E; e0 += 32) {
    const int e = e0 + lane;
    float dp = (dpr && e < E) ? dpr[e] : 0.f;
    for (int k = 0; k < K; ++k) {
      const float dvk = __shfl_sync(0xffffffffu, dv, k);
      const int ek = __shfl_sync(0xffffffffu, myk_e, k);
      if (ek == e) dp += dvk;
    }
    if (e < E) dl[e] = __float2bfloat16_rn(pr[e] * (dp - sdot));
  }
}

int router_bwd(const void* dtopv, bool dtopv_f32, const float* dprobs, const float* probs, const long long* topi,
               const void* per_expert_scale, int T, int E, int K, void* dlogits, long long ld, cudaStream_t st) {
  SMELB_CHECK_ARG(K >= 1 && K <= 32 && E >= K, kErrShape, "router_bwd: E=%d K=%d", E, K);
  if (T == 0) return kOk;
  const int threads = 256;
  router_bwd_kernel<<<(T * 32 + threads - 1) / threads, threads, 0, st>>>(
      dtopv, dtopv_f32 ? 1 : 0, dprobs, probs, topi, (const bf16*)per_expert_scale, T, E, K, (bf16*)dlogits, ld);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

// ============================================================================================ dispatch plan
// Stable counting sort of the flattened expert choices i = t*K + k (a single CTA of 32 warps):
//   counts[e]          number of i with topi[i] == e
//   offsets[e]         first row of expert e in the dispatch layout; selected experts' segments are padded to a
//                      multiple of `pad` rows (zero rows) so LoRA weight-gradient GEMMs can reduce over whole tiles
//   gcounts[e]         rows of expert e's segment (counts, or the padded count for selected experts)
//   row_of[i]          dispatch row of choice i (stable: equal experts keep (t, k) order)
//   src_of[row]        i for real rows, -1 for padding rows (rows < total)
//   order[j]           reference-compatible stable argsort of topi.reshape(-1) (unpadded positions)
//   total[0]           rows used by the dispatch layout
constexpr int kPlanWarps = 32;
constexpr int kPlanMaxE = 512;
constexpr long long kPlanStageMax = 49152;  // choices staged in shared memory as uint16 expert ids

__global__ void __launch_bounds__(kPlanWarps * 32, 1)
    dispatch_plan_kernel(const long long* __restrict__ topi, long long R, int E, const uint8_t* __restrict__ sel_mask,
                         int pad, int* __restrict__ counts, int* __restrict__ gcounts, int* __restrict__ offsets,
                         int* __restrict__ row_of, int* __restrict__ src_of, long long* __restrict__ order,
                         int* __restrict__ total, int* __restrict__ err) {
  extern __shared__ int sm[];
  int* hist = sm;                             // [kPlanWarps][E] per-warp counts, later per-warp running bases
  int* s_off = sm + kPlanWarps * E;           // [E] padded offsets
  int* s_offu = s_off + E;                    // [E] unpadded offsets
  int* s_seg = s_offu + E;                    // [E] padded segment lengths
  int* s_cnt = s_seg + E;                     // [E] counts
  uint16_t* s_eid = reinterpret_cast<uint16_t*>(s_cnt + E);  // [R] expert ids (0xFFFF: invalid), when staged
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool staged = R <= kPlanStageMax;
  for (int i = threadIdx.x; i < kPlanWarps * E; i += blockDim.x) hist[i] = 0;
  if (staged) {
    // coalesced, independent loads: the whole choice list lands in shared memory once
    for (long long i = threadIdx.x; i < R; i += blockDim.x) {
      const long long e = topi[i];
      if (e < 0 || e >= E) dev_fail(err, kDevErrBadIndex);
      s_eid[i] = (e < 0 || e >= E) ? (uint16_t)0xFFFF : (uint16_t)e;
    }
  }
  __syncthreads();
  auto eid = [&](long long i) -> int {
    if (staged) {
      const int e = s_eid[i];
      return e == 0xFFFF ? -1 : e;
    }
    const long long e = topi[i];
    return (e >= 0 && e < E) ? (int)e : -1;
  };
  const long long chunk = (R + kPlanWarps - 1) / kPlanWarps;
  const long long c0 = warp * chunk, c1 = min(R, c0 + chunk);
  for (long long i = c0 + lane; i < c1; i += 32) {
    const int e = eid(i);
    if (e < 0) {
      if (!staged) dev_fail(err, kDevErrBadIndex);
      continue;
    }
    atomicAdd(&hist[warp * E + e], 1);
  }
  __syncthreads();
  // per-expert totals and per-warp exclusive bases
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int w = 0; w < kPlanWarps; ++w) {
      const int c = hist[w * E + e];
      hist[w * E + e] = run;
      run += c;
    }
    counts[e] = run;
    const int seg = (sel_mask && sel_mask[e]) ? (run + pad - 1) / pad * pad : run;
    gcounts[e] = seg;
    s_seg[e] = seg;
    s_cnt[e] = run;
  }
  __syncthreads();
  if (warp == 0) {
    // exclusive scans of the segment lengths and counts: each lane sums a run of consecutive experts
    const int per = (E + 31) / 32;
    const int e0 = lane * per, e1 = min(E, e0 + per);
    int a = 0, au = 0;
    for (int e = e0; e < e1; ++e) {
      a += s_seg[e];
      au += s_cnt[e];
    }
    int ia = a, iau = au;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, ia, o), xu = __shfl_up_sync(0xffffffffu, iau, o);
      if (lane >= o) {
        ia += x;
        iau += xu;
      }
    }
    int acc = ia - a, accu = iau - au;
    for (int e = e0; e < e1; ++e) {
      s_off[e] = acc;
      s_offu[e] = accu;
      acc += s_seg[e];
      accu += s_cnt[e];
    }
    if (lane == 31) total[0] = ia;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) offsets[e] = s_off[e];
  // stable ranks: each warp walks its chunk in order, 32 choices at a time
  const unsigned lt_mask = (1u << lane) - 1u;
  for (long long b = c0; b < c1; b += 32) {
    const long long i = b + lane;
    const int e = i < c1 ? eid(i) : -1;
    const unsigned active = __ballot_sync(0xffffffffu, e >= 0);
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0) {
      const int rank = __popc(peers & active & lt_mask);
      const int pos = hist[warp * E + e] + rank;
      const int row = s_off[e] + pos;
      row_of[i] = row;
      src_of[row] = (int)i;
      order[s_offu[e] + pos] = i;
    }
    __syncwarp();
    if (e >= 0) {
      const int leader = __ffs(peers & active) - 1;
      if (lane == leader) hist[warp * E + e] += __popc(peers & active);
    }
    __syncwarp();
  }
  __syncthreads();
  // padding rows of padded segments
  for (int e = warp; e < E; e += kPlanWarps) {
    const int cnt = s_cnt[e], seg = s_seg[e];
    for (int r = cnt + lane; r < seg; r += 32) src_of[s_off[e] + r] = -1;
  }
}

int dispatch_plan(const long long* topi, long long R, int E, const uint8_t* sel_mask, int pad, int* counts,
                  int* gcounts, int* offsets, int* row_of, int* src_of, long long* order, int* total, cudaStream_t st) {
  SMELB_CHECK_ARG(E >= 1 && E <= kPlanMaxE, kErrShape, "dispatch_plan: E=%d (max %d)", E, kPlanMaxE);
  SMELB_CHECK_ARG(pad >= 1 && R >= 0 && R < (1LL << 30), kErrShape, "dispatch_plan: R=%lld pad=%d", R, pad);
  int dev = 0;
  SMELB_CUDA(cudaGetDevice(&dev));
  const long long staged = R <= kPlanStageMax ? R : 0;
  const int smem = (int)((kPlanWarps * E + 4 * E) * 4 + ((staged * 2 + 15) & ~15LL));
  static bool configured[64] = {false};
  if (dev < 64 && !configured[dev]) {
    SMELB_CUDA(cudaFuncSetAttribute(dispatch_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)((kPlanWarps * kPlanMaxE + 4 * kPlanMaxE) * 4 + kPlanStageMax * 2)));
    configured[dev] = true;
  }
  dispatch_plan_kernel<<<1, kPlanWarps * 32, smem, st>>>(topi, R, E, sel_mask, pad, counts, gcounts, offsets, row_of,
                                                         src_of, order, total, device_status(dev));
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

// Multi-CTA variant of the same plan for callers that can lend scratch (nb x E ints): pass 1 counts each CTA's
// contiguous chunk of choices, pass 2 derives every CTA's base per expert from the earlier chunks' counts, the
// (padded) segment offsets, and then ranks its chunk warp by warp in order, so the result equals the single-CTA plan.
constexpr int kPlanMtWarps = 8;
constexpr long long kPlanMtChunk = 1024;

__global__ void __launch_bounds__(256) plan_count_kernel(const long long* __restrict__ topi, long long R, int E,
                                                         long long chunk, int* __restrict__ cnt, int* __restrict__ err) {
  __shared__ int hist[kPlanMaxE];
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const long long c0 = blockIdx.x * chunk, c1 = min(R, c0 + chunk);
  for (long long i = c0 + threadIdx.x; i < c1; i += blockDim.x) {
    const long long e = topi[i];
    if (e < 0 || e >= E) {
      dev_fail(err, kDevErrBadIndex);
      continue;
    }
    atomicAdd(&hist[(int)e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[(long long)blockIdx.x * E + e] = hist[e];
}

__global__ void __launch_bounds__(kPlanMtWarps * 32) plan_rank_kernel(
    const long long* __restrict__ topi, long long R, int E, long long chunk, const uint8_t* __restrict__ sel_mask,
    int pad, const int* __restrict__ cnt, int* __restrict__ counts, int* __restrict__ gcounts,
    int* __restrict__ offsets, int* __restrict__ row_of, int* __restrict__ src_of, long long* __restrict__ order,
    int* __restrict__ total) {
  __shared__ int base[kPlanMaxE], tot[kPlanMaxE], seg[kPlanMaxE], s_off[kPlanMaxE], s_offu[kPlanMaxE];
  __shared__ int wcnt[kPlanMtWarps][kPlanMaxE];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = gridDim.x, b = blockIdx.x;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    // the column of e over the nb CTAs' counts, 8 loads in flight at a time
    int bs = 0, t = 0;
    for (int bb0 = 0; bb0 < nb; bb0 += 8) {
      int c[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) c[j] = bb0 + j < nb ? cnt[(long long)(bb0 + j) * E + e] : 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        bs += bb0 + j < b ? c[j] : 0;
        t += c[j];
      }
    }
    base[e] = bs;
    tot[e] = t;
    seg[e] = (sel_mask && sel_mask[e]) ? (t + pad - 1) / pad * pad : t;
    for (int w = 0; w < kPlanMtWarps; ++w) wcnt[w][e] = 0;
  }
  __syncthreads();
  if (warp == 0) {
    const int per = (E + 31) / 32;
    const int e0 = lane * per, e1 = min(E, e0 + per);
    int a = 0, au = 0;
    for (int e = e0; e < e1; ++e) {
      a += seg[e];
      au += tot[e];
    }
    int ia = a, iau = au;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, ia, o), xu = __shfl_up_sync(0xffffffffu, iau, o);
      if (lane >= o) {
        ia += x;
        iau += xu;
      }
    }
    int acc = ia - a, accu = iau - au;
    for (int e = e0; e < e1; ++e) {
      s_off[e] = acc;
      s_offu[e] = accu;
      acc += seg[e];
      accu += tot[e];
    }
    if (b == 0 && lane == 31) total[0] = ia;
  }
  // this CTA's chunk, split into kPlanMtWarps consecutive sub-chunks
  const long long c0 = b * chunk, c1 = min(R, c0 + chunk);
  const long long sub = (c1 - c0 + kPlanMtWarps - 1) / kPlanMtWarps;
  const long long w0 = min(c1, c0 + warp * sub), w1 = min(c1, w0 + sub);
  for (long long i = w0 + lane; i < w1; i += 32) {
    const long long e = topi[i];
    if (e >= 0 && e < E) atomicAdd(&wcnt[warp][(int)e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    if (b == 0) {
      counts[e] = tot[e];
      gcounts[e] = seg[e];
      offsets[e] = s_off[e];
    }
    int run = base[e];
    for (int w = 0; w < kPlanMtWarps; ++w) {
      const int c = wcnt[w][e];
      wcnt[w][e] = run;
      run += c;
    }
  }
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  long long e_next = w0 + lane < w1 ? topi[w0 + lane] : -1;  // the next round's choice, loaded a round ahead
  for (long long r0 = w0; r0 < w1; r0 += 32) {
    const long long i = r0 + lane;
    const long long e64 = e_next;
    e_next = r0 + 32 + lane < w1 ? topi[r0 + 32 + lane] : -1;
    const int e = (e64 >= 0 && e64 < E) ? (int)e64 : -1;
    const unsigned active = __ballot_sync(0xffffffffu, e >= 0);
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0) {
      const int pos = wcnt[warp][e] + __popc(peers & active & lt_mask);
      const int row = s_off[e] + pos;
      row_of[i] = row;
      src_of[row] = (int)i;
      order[s_offu[e] + pos] = i;
    }
    __syncwarp();
    if (e >= 0 && lane == __ffs(peers & active) - 1) wcnt[warp][e] += __popc(peers & active);
    __syncwarp();
  }
  // padding rows of the padded segments of this CTA's experts
  for (int e = b; e < E; e += nb)
    for (int r = tot[e] + threadIdx.x; r < seg[e]; r += blockDim.x) src_of[s_off[e] + r] = -1;
}

int dispatch_plan_mt(const long long* topi, long long R, int E, const uint8_t* sel_mask, int pad, int* counts,
                     int* gcounts, int* offsets, int* row_of, int* src_of, long long* order, int* total, int* scratch,
                     long long scratch_ints, cudaStream_t st) {
  SMELB_CHECK_ARG(E >= 1 && E <= kPlanMaxE, kErrShape, "dispatch_plan: E=%d (max %d)", E, kPlanMaxE);
  SMELB_CHECK_ARG(pad >= 1 && R >= 0 && R < (1LL << 30), kErrShape, "dispatch_plan: R=%lld pad=%d", R, pad);
  // CTAs: every CTA sums the counts of the CTAs before it, one dependent L2 round trip per 8 of them, so fewer CTAs
  // with more choices each (about 1024) finish sooner than one CTA per SM (32768 choices: 11 us at 127 CTAs)
  long long nb = R / 256 < 2 ? 1 : std::min<long long>(148, std::max<long long>(2, R / kPlanMtChunk));
  nb = std::min<long long>(nb, scratch_ints / E);
  if (nb < 2) return dispatch_plan(topi, R, E, sel_mask, pad, counts, gcounts, offsets, row_of, src_of, order, total, st);
  const long long chunk = (R + nb - 1) / nb;
  int dev = 0;
  SMELB_CUDA(cudaGetDevice(&dev));
  plan_count_kernel<<<(int)nb, 256, 0, st>>>(topi, R, E, chunk, scratch, device_status(dev));
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  plan_rank_kernel<<<(int)nb, kPlanMtWarps * 32, 0, st>>>(topi, R, E, chunk, sel_mask, pad, scratch, counts, gcounts,
                                                          offsets, row_of, src_of, order, total);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

// ============================================================================================ row norms
// RMSNorm of bf16 rows in fp32 (smel/norm.py:1-20 and its torch form smel/layer_runner.py:110-130), one warp per row:
//   v = x, or with a residual input h: s = bf16(h + x) (stored) and v = s;
//   rstd = rsqrt(mean(v^2) + eps);  y = bf16(v * rstd * w')  with w' = 1 (w_mode 0), w (1) or 1 + w (2).
// The Gemma 4 router prologue (smel/moe.py:170-176) is w_mode 0 plus a post chain in the reference's bf16 steps:
//   y = bf16(bf16(bf16(v * rstd) * scale[c]) * post_mul)   (post_scale != null and/or post_mul != 0).
// Backward (frozen norm weights): g = dy * w' (with the post chain: g = bf16(bf16(dy * post_mul) * scale)),
//   dx = rstd * (g - xhat * mean(g * xhat)) [+ ds], xhat = v * rstd.
__device__ __forceinline__ void ld8(const bf16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* q = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(q[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}
__device__ __forceinline__ void st8(bf16* p, const float (&v)[8]) {
  uint4 u;
  __nv_bfloat162* q = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) q[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ float weff(const bf16* w, int w_mode, int c) {
  if (w_mode == 0) return 1.f;
  const float f = __bfloat162float(w[c]);
  return w_mode == 2 ? 1.f + f : f;
}

__global__ void rmsnorm_fwd_kernel(const NormArgs a) {
  const int lane = threadIdx.x & 31;
  const long long nw = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; r < a.rows; r += nw) {
    const long long o = r * a.C;
    float ss = 0.f;
    for (int c = lane * 8; c < a.C; c += 256) {
      float v[8];
      ld8(a.x + o + c, v);
      if (a.h) {
        float hv[8];
        ld8(a.h + o + c, hv);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = bf16_round(hv[j] + v[j]);  // the residual stream is rounded
        st8(a.s + o + c, v);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(v[j], v[j], ss);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float rs = rsqrtf(ss / (float)a.C + a.eps);
    if (a.rstd && lane == 0) a.rstd[r] = rs;
    const bf16* src = a.h ? a.s : a.x;
    for (int c = lane * 8; c < a.C; c += 256) {
      float v[8];
      ld8(src + o + c, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float y = v[j] * rs * weff(a.w, a.w_mode, c + j);
        if (a.post_scale) y = bf16_round(bf16_round(y) * __bfloat162float(a.post_scale[c + j]));
        if (a.post_mul != 0.f) y = bf16_round(y) * a.post_mul;
        v[j] = y;
      }
      st8(a.y + o + c, v);
    }
  }
}

__global__ void rmsnorm_bwd_kernel(const NormBwdArgs a) {
  const int lane = threadIdx.x & 31;
  const long long nw = (long long)gridDim.x * (blockDim.x >> 5);
  auto gval = [&](float dy, int c) {
    float g = dy;
    if (a.post_mul != 0.f) g = bf16_round(g * a.post_mul);
    if (a.post_scale) g = bf16_round(g * __bfloat162float(a.post_scale[c]));
    return g * weff(a.w, a.w_mode, c);
  };
  for (long long r = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; r < a.rows; r += nw) {
    const long long o = r * a.C;
    const float rs = a.rstd[r];
    float dot = 0.f;
    for (int c = lane * 8; c < a.C; c += 256) {
      float d[8], v[8];
      ld8(a.dy + o + c, d);
      ld8(a.x + o + c, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) dot = fmaf(gval(d[j], c + j), v[j] * rs, dot);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    const float mc = dot / (float)a.C;
    for (int c = lane * 8; c < a.C; c += 256) {
      float d[8], v[8], e[8];
      ld8(a.dy + o + c, d);
      ld8(a.x + o + c, v);
      if (a.ds) ld8(a.ds + o + c, e);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float dx = rs * (gval(d[j], c + j) - v[j] * rs * mc);
        if (a.ds) dx += e[j];
        d[j] = dx;
      }
      st8(a.dx + o + c, d);
    }
  }
}

int rmsnorm_fwd(const NormArgs& a, cudaStream_t st) {
  SMELB_CHECK_ARG(a.C % 8 == 0 && a.C > 0, kErrShape, "rmsnorm: %d columns (a multiple of 8)", a.C);
  SMELB_CHECK_ARG(!a.h || a.s, kErrArg, "rmsnorm: the fused add needs its sum output");
  SMELB_CHECK_ARG(a.w_mode == 0 || a.w, kErrArg, "rmsnorm: w_mode %d without a weight", a.w_mode);
  if (a.rows == 0) return kOk;
  const long long blocks = std::min<long long>((a.rows * 32 + 255) / 256, 148LL * 16);
  rmsnorm_fwd_kernel<<<(int)blocks, 256, 0, st>>>(a);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

int rmsnorm_bwd(const NormBwdArgs& a, cudaStream_t st) {
  SMELB_CHECK_ARG(a.C % 8 == 0 && a.C > 0, kErrShape, "rmsnorm_bwd: %d columns (a multiple of 8)", a.C);
  SMELB_CHECK_ARG(a.w_mode == 0 || a.w, kErrArg, "rmsnorm_bwd: w_mode %d without a weight", a.w_mode);
  if (a.rows == 0) return kOk;
  const long long blocks = std::min<long long>((a.rows * 32 + 255) / 256, 148LL * 16);
  rmsnorm_bwd_kernel<<<(int)blocks, 256, 0, st>>>(a);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

// CTAs of one full wave of a grid-stride kernel (every SM at its occupancy limit): launched with this many, the CTAs
// loop over the units with no partly filled tail wave (a grid of 1184 CTAs at 6 resident per SM is 1.33 waves).
template <class Kern>
long long one_wave(Kern kernel, int threads) {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, 0) != cudaSuccess || n < 1) n = 1;
  return (long long)num_sms(dev) * n;
}

// ============================================================================================ gather
// xs[row] = x[src_of[row] / K] for real rows and zeros for padding rows, rows < total[0]. One warp per row, 16-byte
// vectors (H % 8 == 0).
__global__ void gather_rows_kernel(const bf16* __restrict__ x, int H, int K, const int* __restrict__ src_of,
                                   const int* __restrict__ total, long long max_rows, bf16* __restrict__ xs) {
  const long long rows = min((long long)total[0], max_rows);
  const int lane = threadIdx.x & 31;
  const long long nw = (long long)gridDim.x * (blockDim.x >> 5);
  const int nv = H / 8;
  for (long long r = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; r < rows; r += nw) {
    const int src = src_of[r];
    uint4* dst = reinterpret_cast<uint4*>(xs + r * H);
    if (src < 0) {
      for (int v = lane; v < nv; v += 32) dst[v] = make_uint4(0, 0, 0, 0);
    } else {
      const uint4* s = reinterpret_cast<const uint4*>(x + (long long)(src / K) * H);
      for (int v = lane; v < nv; v += 32) dst[v] = __ldg(s + v);
    }
  }
}

int gather_rows(const void* x, int H, int K, const int* src_of, const int* total, long long max_rows, void* xs,
                cudaStream_t st) {
  SMELB_CHECK_ARG(H % 8 == 0, kErrShape, "gather_rows: H=%d not a multiple of 8", H);
  if (max_rows == 0) return kOk;
  const int threads = 256;
  const long long blocks = std::min<long long>((max_rows * 32 + threads - 1) / threads, 148LL * 8);
  gather_rows_kernel<<<(int)blocks, threads, 0, st>>>((const bf16*)x, H, K, src_of, total, max_rows, (bf16*)xs);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

// ============================================================================================ combine
// out[t] = bf16( sum_k fl(y[row_of[t,k]] * topv[t,k]) ) accumulated in fp32 in k order; with a shared expert:
// out[t] = bf16( that + bf16(y_sh[t] * bf16(sigmoid(gl[t]))) ) (the reference's bf16 op sequence). One warp per
// (token, 256-column block), 8 columns per lane; a block's K expert rows are loaded together before they are summed
// (in k order), so a few tokens still keep many loads in flight.
// One warp per unit = (token, slice of nch 256-column chunks): the unit's K row indices and weights are loaded once
// (eight at a time), then each chunk's eight rows are loaded together and summed in k order. The slice is the whole
// row when there are enough tokens to fill the GPU and shrinks to one chunk for a handful of tokens (decode).
#ifndef SMELB_COMBINE_CHUNKS
#define SMELB_COMBINE_CHUNKS 2
#endif
constexpr int kCombineMaxChunks = SMELB_COMBINE_CHUNKS;

__global__ void combine_fwd_kernel(const bf16* __restrict__ y, const int* __restrict__ row_of,
                                   const void* __restrict__ topv, int topv_f32, int T, int K, int H, int nch,
                                   const bf16* __restrict__ y_sh, const bf16* __restrict__ gl, int has_routed,
                                   bf16* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int chunks = (H + 255) / 256;
  const int nsl = (chunks + nch - 1) / nch;  // slices per token
  const long long nw = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long u = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; u < (long long)T * nsl; u += nw) {
    const long long t = u / nsl;
    const int ch0 = (int)(u - t * nsl) * nch;
    float acc[kCombineMaxChunks][8];
#pragma unroll
    for (int q = 0; q < kCombineMaxChunks; ++q)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[q][j] = 0.f;
    if (has_routed) {
      for (int k0 = 0; k0 < K; k0 += 8) {
        float w[8];
        int rows[8];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const long long o = t * K + k0 + kk;
          const bool in = k0 + kk < K;
          w[kk] = !in ? 0.f
                      : topv_f32 ? reinterpret_cast<const float*>(topv)[o]
                                 : __bfloat162float(reinterpret_cast<const bf16*>(topv)[o]);
          rows[kk] = in ? row_of[o] : 0;
        }
#pragma unroll
        for (int q = 0; q < kCombineMaxChunks; ++q) {
          const int c = (ch0 + q) * 256 + lane * 8;
          if (q >= nch || c >= H) break;
          uint4 v[8];
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            if (k0 + kk < K) v[kk] = *reinterpret_cast<const uint4*>(y + (long long)rows[kk] * H + c);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            if (k0 + kk < K) {
              const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v[kk]);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float2 f = __bfloat1622float2(p[j]);
                acc[q][2 * j] = __fadd_rn(acc[q][2 * j], __fmul_rn(f.x, w[kk]));
                acc[q][2 * j + 1] = __fadd_rn(acc[q][2 * j + 1], __fmul_rn(f.y, w[kk]));
              }
            }
          }
        }
      }
    }
    float sg = 0.f;
    if (y_sh && gl) {
      const float g = __bfloat162float(gl[t]);
      sg = bf16_round(1.0f / (1.0f + expf(-g)));
    }
#pragma unroll
    for (int q = 0; q < kCombineMaxChunks; ++q) {
      const int c = (ch0 + q) * 256 + lane * 8;
      if (q >= nch || c >= H) break;
      float res[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) res[j] = bf16_round(acc[q][j]);
      if (y_sh) {
        const uint4 v = *reinterpret_cast<const uint4*>(y_sh + t * H + c);
        const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(p[j]);
          const float a = gl ? bf16_round(f.x * sg) : f.x;
          const float b = gl ? bf16_round(f.y * sg) : f.y;
          res[2 * j] = has_routed ? res[2 * j] + a : a;
          res[2 * j + 1] = has_routed ? res[2 * j + 1] + b : b;
        }
      }
      uint4 o;
      __nv_bfloat162* po = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) po[j] = __floats2bfloat162_rn(res[2 * j], res[2 * j + 1]);
      *reinterpret_cast<uint4*>(out + t * H + c) = o;
    }
  }
}

int combine_fwd(const void* y, const int* row_of, const void* topv, bool topv_f32, int T, int K, int H,
                const void* y_sh, const void* gl, void* out, cudaStream_t st) {
  SMELB_CHECK_ARG(H % 8 == 0 && K <= 32, kErrShape, "combine_fwd: H=%d K=%d", H, K);
  if (T == 0) return kOk;
  const int threads = 256;
  const int chunks = (H + 255) / 256;
  // chunks per unit: as many as keep at least ~8 warps per SM busy, at most kCombineMaxChunks (2: at 4092 tokens 1
  // chunk per unit ran 15% slower, 4 chunks need 128 registers and half the warps per SM and ran 5% slower)
  int nch = kCombineMaxChunks;
  while (nch > 1 && (long long)T * ((chunks + nch - 1) / nch) < 148LL * 8) nch >>= 1;
  nch = std::min(nch, chunks);
  const long long units = (long long)T * ((chunks + nch - 1) / nch);
  static const long long wave = one_wave(combine_fwd_kernel, threads);
  const long long blocks = std::min<long long>((units * 32 + threads - 1) / threads, wave);
  combine_fwd_kernel<<<(int)blocks, threads, 0, st>>>((const bf16*)y, row_of, topv, topv_f32 ? 1 : 0, T, K, H, nch,
                                                      (const bf16*)y_sh, (const bf16*)gl, y != nullptr ? 1 : 0,
                                                      (bf16*)out);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

// Backward of the combine, one warp per dispatch row (rows < total):
//   dy[row] = bf16(g[t] * topv[t,k]); dtopv[t,k] = sum_h g[t,h] * y[row,h] (fp32, stored in topv's dtype);
//   padding rows get dy = 0.
__global__ void combine_bwd_rows_kernel(const bf16* __restrict__ g, const bf16* __restrict__ y,
                                        const int* __restrict__ src_of, const int* __restrict__ total,
                                        long long max_rows, const void* __restrict__ topv, int topv_f32, int K, int H,
                                        bf16* __restrict__ dy, void* __restrict__ dtopv) {
  const long long rows = min((long long)total[0], max_rows);
  const int lane = threadIdx.x & 31;
  const long long nw = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; r < rows; r += nw) {
    const int src = src_of[r];
    uint4* d = reinterpret_cast<uint4*>(dy + r * H);
    if (src < 0) {
      for (int c = lane; c < H / 8; c += 32) d[c] = make_uint4(0, 0, 0, 0);
      continue;
    }
    const long long t = src / K;
    const float w = topv_f32 ? reinterpret_cast<const float*>(topv)[src]
                             : __bfloat162float(reinterpret_cast<const bf16*>(topv)[src]);
    float dot = 0.f;
    // four 16-byte pieces of g and y per lane are loaded before any is used (the dot product keeps its order)
    for (int c0 = lane; c0 < H / 8; c0 += 128) {
      uint4 gv[4], yv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (c0 + 32 * q < H / 8) {
          gv[q] = reinterpret_cast<const uint4*>(g + t * H)[c0 + 32 * q];
          yv[q] = reinterpret_cast<const uint4*>(y + r * H)[c0 + 32 * q];
        }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (c0 + 32 * q >= H / 8) break;
        const __nv_bfloat162* gp = reinterpret_cast<const __nv_bfloat162*>(&gv[q]);
        const __nv_bfloat162* yp = reinterpret_cast<const __nv_bfloat162*>(&yv[q]);
        uint4 o;
        __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 gf = __bfloat1622float2(gp[j]);
          const float2 yf = __bfloat1622float2(yp[j]);
          op[j] = __floats2bfloat162_rn(gf.x * w, gf.y * w);
          dot = fmaf(gf.x, yf.x, dot);
          dot = fmaf(gf.y, yf.y, dot);
        }
        d[c0 + 32 * q] = o;
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if (lane == 0 && dtopv) {
      if (topv_f32) reinterpret_cast<float*>(dtopv)[src] = dot;
      else reinterpret_cast<bf16*>(dtopv)[src] = __float2bfloat16_rn(dot);
    }
  }
}

int combine_bwd_rows(const void* g, const void* y, const int* src_of, const int* total, long long max_rows,
                     const void* topv, bool topv_f32, int K, int H, void* dy, void* dtopv, cudaStream_t st) {
  SMELB_CHECK_ARG(H % 8 == 0, kErrShape, "combine_bwd: H=%d", H);
  if (max_rows == 0) return kOk;
  const int threads = 256;
  static const long long wave = one_wave(combine_bwd_rows_kernel, threads);
  const long long blocks = std::min<long long>((max_rows * 32 + threads - 1) / threads, wave);
  combine_bwd_rows_kernel<<<(int)blocks, threads, 0, st>>>((const bf16*)g, (const bf16*)y, src_of, total, max_rows,
                                                           topv, topv_f32 ? 1 : 0, K, H, (bf16*)dy, dtopv);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

// Shared expert gate backward, one warp per token: dy_sh = bf16(g * s_b) with s_b = bf16(sigmoid(gl));
// ds = sum_h g * y_sh (fp32); dgl = ds * s_b * (1 - s_b), stored as fp32 for the final dX reduction.
__global__ void shared_gate_bwd_kernel(const bf16* __restrict__ g, const bf16* __restrict__ y_sh,
                                       const bf16* __restrict__ gl, int T, int H, bf16* __restrict__ dy_sh,
                                       float* __restrict__ dgl) {
  const int lane = threadIdx.x & 31;
  const long long nw = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long t = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; t < T; t += nw) {
    const float sb = bf16_round(1.0f / (1.0f + expf(-__bfloat162float(gl[t]))));
    float dot = 0.f;
    for (int c0 = lane; c0 < H / 8; c0 += 128) {
      uint4 gv[4], yv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (c0 + 32 * q < H / 8) {
          gv[q] = reinterpret_cast<const uint4*>(g + t * H)[c0 + 32 * q];
          yv[q] = reinterpret_cast<const uint4*>(y_sh + t * H)[c0 + 32 * q];
        }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (c0 + 32 * q >= H / 8) break;
        const __nv_bfloat162* gp = reinterpret_cast<const __nv_bfloat162*>(&gv[q]);
        const __nv_bfloat162* yp = reinterpret_cast<const __nv_bfloat162*>(&yv[q]);
        uint4 o;
        __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 gf = __bfloat1622float2(gp[j]);
          const float2 yf = __bfloat1622float2(yp[j]);
          op[j] = __floats2bfloat162_rn(gf.x * sb, gf.y * sb);
          dot = fmaf(gf.x, yf.x, dot);
          dot = fmaf(gf.y, yf.y, dot);
        }
        reinterpret_cast<uint4*>(dy_sh + t * H)[c0 + 32 * q] = o;
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if (lane == 0) dgl[t] = bf16_round(bf16_round(dot) * sb * (1.0f - sb));
  }
}

int shared_gate_bwd(const void* g, const void* y_sh, const void* gl, int T, int H, void* dy_sh, float* dgl,
                    cudaStream_t st) {
  if (T == 0) return kOk;
  const int threads = 256;
  const long long blocks = std::min<long long>(((long long)T * 32 + threads - 1) / threads, 148LL * 8);
  shared_gate_bwd_kernel<<<(int)blocks, threads, 0, st>>>((const bf16*)g, (const bf16*)y_sh, (const bf16*)gl, T, H,
                                                          (bf16*)dy_sh, dgl);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

// Final dX of the layer, fp32 accumulation then one rounding:
//   dx[t] = sum_k dxs[row_of[t,k]] + dx_sh[t] + dx_r[t] + dgl[t] * w_sg
// One warp per (token, 256-column chunk), 8 columns per lane: a warp loads the token's row ids (one broadcast load
// each), then eight rows' 16-byte pieces together, and adds them in k order. Small units keep many warps resident
// (a warp per whole token, walking its 2048 columns in eight dependent steps, moved the bytes at about half of HBM).
__global__ void __launch_bounds__(256) dx_reduce_kernel(const bf16* __restrict__ dxs, const int* __restrict__ row_of,
                                                        int K, int T, int H, const bf16* __restrict__ dx_sh,
                                                        const bf16* __restrict__ dx_r, const float* __restrict__ dgl,
                                                        const bf16* __restrict__ w_sg, bf16* __restrict__ dx) {
  const int lane = threadIdx.x & 31;
  const int chunks = (H + 255) / 256;
  const long long units = (long long)T * chunks;
  const long long nw = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long u = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; u < units; u += nw) {
    const long long t = u / chunks;
    const int c = (int)(u - t * chunks) * 256 + lane * 8;
    if (c >= H) continue;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    auto add = [&](const uint4& v) {
      const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(p[j]);
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    };
    if (dxs) {
      for (int k0 = 0; k0 < K; k0 += 8) {
        int rows[8];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) rows[kk] = k0 + kk < K ? row_of[t * K + k0 + kk] : 0;
        uint4 v[8];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          if (k0 + kk < K) v[kk] = *reinterpret_cast<const uint4*>(dxs + (long long)rows[kk] * H + c);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          if (k0 + kk < K) add(v[kk]);
      }
    }
    if (dx_sh) add(*reinterpret_cast<const uint4*>(dx_sh + t * H + c));
    if (dx_r) add(*reinterpret_cast<const uint4*>(dx_r + t * H + c));
    if (dgl && w_sg) {
      const float dg = dgl[t];
      const uint4 v = *reinterpret_cast<const uint4*>(w_sg + c);
      const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(p[j]);
        acc[2 * j] = fmaf(dg, f.x, acc[2 * j]);
        acc[2 * j + 1] = fmaf(dg, f.y, acc[2 * j + 1]);
      }
    }
    uint4 o;
    __nv_bfloat162* po = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) po[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
    *reinterpret_cast<uint4*>(dx + t * H + c) = o;
  }
}

int dx_reduce(const void* dxs, const int* row_of, int K, int T, int H, const void* dx_sh, const void* dx_r,
              const float* dgl, const void* w_sg, void* dx, cudaStream_t st) {
  SMELB_CHECK_ARG(H % 8 == 0 && K <= 32, kErrShape, "dx_reduce: H=%d K=%d", H, K);
  if (T == 0) return kOk;
  const int threads = 256;
  const long long units = (long long)T * ((H + 255) / 256);
  static const long long wave = one_wave(dx_reduce_kernel, threads);
  const long long blocks = std::min<long long>((units * 32 + threads - 1) / threads, wave);
  dx_reduce_kernel<<<(int)blocks, threads, 0, st>>>((const bf16*)dxs, row_of, K, T, H, (const bf16*)dx_sh,
                                                    (const bf16*)dx_r, dgl, (const bf16*)w_sg, (bf16*)dx);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

// ============================================================================================ LoRA factor packing
// out[j][a][b] (bf16, J x OA x OB) = scale_i * src_i[j*sj + (a - a0)*sa + (b - b0)*sb] inside block i (two blocks),
// zero elsewhere. Used to build the per-step bf16 operands of the LoRA GEMMs from the fp32 parameters
// (concatenations, block-diagonal stacks, transposes, scale folding and zero padding to 64 columns).
__global__ void pack_blocks_kernel(PackSpec spec, bf16* __restrict__ out) {
  const long long n = (long long)spec.J * spec.OA * spec.OB;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long j = i / ((long long)spec.OA * spec.OB);
    const long long rem = i - j * spec.OA * spec.OB;
    const int a = (int)(rem / spec.OB), b = (int)(rem - (long long)a * spec.OB);
    float v = 0.f;
#pragma unroll
    for (int bi = 0; bi < 2; ++bi) {
      const PackBlock& B = spec.blk[bi];
      if (B.src && a >= B.a0 && a < B.a0 + B.na && b >= B.b0 && b < B.b0 + B.nb)
        v = B.scale * B.src[j * B.sj + (long long)(a - B.a0) * B.sa + (long long)(b - B.b0) * B.sb];
    }
    out[i] = __float2bfloat16_rn(v);
  }
}

__device__ __forceinline__ uint32_t pk_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }
// One thread per 8 consecutive outputs of a row (j, a) of one of the batch's outputs (OB % 8 == 0): the block
// descriptions are read once per thread into registers and the 8 values leave as one 16-byte store.
__global__ void pack_batch_kernel(const __grid_constant__ PackBatch b) {
  const long long nvec = b.start[b.n] / 8;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < nvec; t += (long long)gridDim.x * blockDim.x) {
    const long long i = t * 8;
    int k = 0;
    while (k + 1 < b.n && i >= b.start[k + 1]) ++k;
    const int OA = b.spec[k].OA, OB = b.spec[k].OB;
    const long long li = i - b.start[k];
    const int row = (int)(li / OB), c0 = (int)(li - (long long)row * OB);
    const int j = row / OA, a = row - j * OA;
    float v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) v[q] = 0.f;
#pragma unroll
    for (int bi = 0; bi < 2; ++bi) {
      const PackBlock B = b.spec[k].blk[bi];
      if (!B.src || a < B.a0 || a >= B.a0 + B.na) continue;
      const float* src = B.src + j * B.sj + (long long)(a - B.a0) * B.sa;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int c = c0 + q;
        if (c >= B.b0 && c < B.b0 + B.nb) v[q] = B.scale * src[(long long)(c - B.b0) * B.sb];
      }
    }
    uint4 o;
    o.x = pk_bits(__floats2bfloat162_rn(v[0], v[1]));
    o.y = pk_bits(__floats2bfloat162_rn(v[2], v[3]));
    o.z = pk_bits(__floats2bfloat162_rn(v[4], v[5]));
    o.w = pk_bits(__floats2bfloat162_rn(v[6], v[7]));
    *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(b.out[k]) + li) = o;
  }
}

int pack_batch(PackBatch& b, cudaStream_t st) {
  b.start[0] = 0;
  b.rstart[0] = 0;
  for (int k = 0; k < b.n; ++k) {
    b.start[k + 1] = b.start[k] + (long long)b.spec[k].J * b.spec[k].OA * b.spec[k].OB;
    b.rstart[k + 1] = b.rstart[k] + b.spec[k].J * b.spec[k].OA;
  }
  if (b.n == 0 || b.start[b.n] == 0) return kOk;
  for (int k = 0; k < b.n; ++k)
    SMELB_CHECK_ARG(b.spec[k].OB % 8 == 0 && (reinterpret_cast<uintptr_t>(b.out[k]) & 15) == 0, kErrShape,
                    "pack: output %d row length %d (needs a multiple of 8, 16-byte aligned)", k, b.spec[k].OB);
  const long long nvec = b.start[b.n] / 8;
  const int blocks = (int)std::min<long long>(148 * 8, (nvec + 255) / 256);
  pack_batch_kernel<<<blocks, 256, 0, st>>>(b);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

int pack_blocks(const PackSpec& spec, void* out, cudaStream_t st) {
  const long long n = (long long)spec.J * spec.OA * spec.OB;
  if (n == 0) return kOk;
  const long long blocks = std::min<long long>((n + 255) / 256, 148LL * 8);
  pack_blocks_kernel<<<(int)blocks, 256, 0, st>>>(spec, (bf16*)out);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}


// ============================================================================================ chunked CE
// The per-row steps of smel/loss.py:50-92 (_ce_chunk) for one vocabulary chunk, in the reference's order: the
// (capped) logits z, the chunk maximum, the new running maximum nm and the rescale r = exp(m - nm), the softmax
// numerators exp(z - nm) summed into s = s * r + sum, then (for the gradient) multiplied by the cap's derivative
// 1 - (z / cap)^2 and rounded to bf16 as the reference's p.to(h.dtype). The target's logit, the cap's derivative
// there and its head row are taken from the chunk that holds the target.
__device__ __forceinline__ float ce_cap(float z, float cap) { return cap > 0.f ? cap * tanhf(z / cap) : z; }

template <bool kMax>
__device__ __forceinline__ float block_reduce_256(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = kMax ? fmaxf(v, u) : v + u;
  }
  __syncthreads();  // red may still be read by the previous reduction
  if (lane == 0) red[w] = v;
  __syncthreads();
  v = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) v = kMax ? fmaxf(v, red[i]) : v + red[i];
  return v;
}

// p[i] = min(step, total - i * step) for the nchunks chunks of `total` rows (the device-side token counts the GEMMs read)
__global__ void set_counts_kernel(int* p, int nchunks, int step, long long total) {
  for (int i = threadIdx.x; i < nchunks; i += blockDim.x)
    p[i] = (int)std::min<long long>(step, total - (long long)i * step);
}

__global__ void ce_init_kernel(CeState st, long long n, int H) {
  const long long tot = st.acc ? n * H : n;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < tot; i += (long long)gridDim.x * blockDim.x) {
    if (st.acc) {
      st.acc[i] = 0.f;
      st.tgt_row[i] = 0.f;
    }
    if (i < n) {
      st.m[i] = -INFINITY;
      st.s[i] = 0.f;
      st.r[i] = 0.f;
      st.tlog[i] = 0.f;
      st.tdrv[i] = 1.f;
    }
  }
}

// One block per token row; 16-byte accesses (ld is a multiple of 64, the rows 128-byte aligned). The row's logits
// are read twice (maximum, then exponentials) and overwritten in place by p. The cap is monotonic, so the chunk
// maximum of the capped logits is the cap of the raw maximum.
__global__ void __launch_bounds__(256) ce_rows_kernel(bf16* __restrict__ lg, int ld, int Vc, long long v0,
                                                     const long long* __restrict__ tgt, float cap, int need_grad,
                                                     const bf16* __restrict__ wc, int H, CeState st) {
  __shared__ float red[8];
  const long long row = blockIdx.x;
  bf16* l = lg + row * ld;
  uint4* lv = reinterpret_cast<uint4*>(l);
  const int nvec = ld >> 3;
  const long long t = tgt[row];
  const bool has_t = t >= v0 && t < v0 + Vc;
  const int c = has_t ? (int)(t - v0) : 0;
  const float zt = has_t ? ce_cap(__bfloat162float(l[c]), cap) : 0.f;  // read before any thread writes p
  float raw = -INFINITY;
  for (int j = threadIdx.x; j < nvec; j += 256) {
    const uint4 u = lv[j];
    const bf16* b = reinterpret_cast<const bf16*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (8 * j + e < Vc) raw = fmaxf(raw, __bfloat162float(b[e]));
  }
  raw = block_reduce_256<true>(raw, red);
  const float cm = ce_cap(raw, cap);
  const float m_old = st.m[row];
  const float nm = fmaxf(m_old, cm);
  const float r = expf(m_old - nm);
  float sum = 0.f;
  for (int j = threadIdx.x; j < nvec; j += 256) {
    const uint4 u = lv[j];
    const bf16* b = reinterpret_cast<const bf16*>(&u);
    uint4 o;
    __nv_bfloat162* ow = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      float pv[2];
#pragma unroll
      for (int f = 0; f < 2; ++f) {
        pv[f] = 0.f;
        if (8 * j + e + f < Vc) {
          const float z = ce_cap(__bfloat162float(b[e + f]), cap);
          const float ex = expf(z - nm);
          sum += ex;
          pv[f] = cap > 0.f ? ex * (1.f - (z / cap) * (z / cap)) : ex;
        }
      }
      ow[e >> 1] = __floats2bfloat162_rn(pv[0], pv[1]);
    }
    if (need_grad) lv[j] = o;
  }
  sum = block_reduce_256<false>(sum, red);
  if (threadIdx.x == 0) {
    st.s[row] = st.s[row] * r + sum;
    st.m[row] = nm;
    st.r[row] = r;
    if (has_t) {
      st.tlog[row] = zt;
      if (cap > 0.f) st.tdrv[row] = 1.f - (zt / cap) * (zt / cap);
    }
  }
  if (has_t && need_grad)
    for (int i = threadIdx.x; i < H; i += 256) st.tgt_row[row * H + i] = __bfloat162float(wc[(long long)c * H + i]);
}

// float4 over [n, H] (H % 4 == 0; the arrays are 16-byte aligned)
__global__ void ce_acc_kernel(const float4* __restrict__ parts, int nparts, CeState st, long long n, int H) {
  const int h4 = H >> 2;
  const long long tot4 = n * h4;
  float4* acc = reinterpret_cast<float4*>(st.acc);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < tot4; i += (long long)gridDim.x * blockDim.x) {
    float4 pw = parts[i];
    for (int q = 1; q < nparts; ++q) {
      const float4 u = parts[q * tot4 + i];
      pw.x += u.x;
      pw.y += u.y;
      pw.z += u.z;
      pw.w += u.w;
    }
    const float r = st.r[i / h4];
    float4 a = acc[i];
    a.x = a.x * r + pw.x;
    a.y = a.y * r + pw.y;
    a.z = a.z * r + pw.z;
    a.w = a.w * r + pw.w;
    acc[i] = a;
  }
}

__global__ void ce_finish_kernel(CeState st, long long n, int H, float denom, float* __restrict__ loss_rows,
                                 bf16* __restrict__ gh) {
  const long long tot = n * H;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < tot; i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / H;
    if (gh) gh[i] = __float2bfloat16_rn((st.acc[i] / st.s[row] - st.tdrv[row] * st.tgt_row[i]) / denom);
    if (i < n) loss_rows[i] = st.m[i] + logf(st.s[i]) - st.tlog[i];
  }
}

__global__ void __launch_bounds__(256) ce_loss_sum_kernel(const float* __restrict__ loss_rows, long long n,
                                                         float denom, float* __restrict__ loss) {
  __shared__ float red[8];
  float v = 0.f;
  for (long long i = threadIdx.x; i < n; i += 256) v += loss_rows[i];
  v = block_reduce_256<false>(v, red);
  if (threadIdx.x == 0) *loss = v / denom;
}

template <typename OutT>
__global__ void int8_rows_dequant_kernel(const int8_t* __restrict__ q, const bf16* __restrict__ scale,
                                         long long rows, int H, OutT* __restrict__ out) {
  const long long tot = rows * H;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < tot; i += (long long)gridDim.x * blockDim.x) {
    const float v = (float)q[i] * __bfloat162float(scale[i / H]);  // exact in fp32 (8-bit times 8-bit mantissas)
    if constexpr (std::is_same<OutT, float>::value) out[i] = v;
    else out[i] = __float2bfloat16_rn(v);
  }
}

__global__ void ce_logits_out_kernel(const bf16* __restrict__ lg, int ld, int Vc, long long n, float cap,
                                     float* __restrict__ out, long long ldo) {
  const long long tot = n * Vc;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < tot; i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / Vc;
    const int v = (int)(i - row * Vc);
    out[row * ldo + v] = ce_cap(__bfloat162float(lg[row * ld + v]), cap);
  }
}

// smel/quant.py:97-101: s = max(amax|w| / 127, 1e-12) in fp32, q = clamp(rint(w / s), -127, 127) (round half to
// even, as torch.round), the scale stored as bf16. One block per row.
__global__ void __launch_bounds__(256) int8_rows_quantize_kernel(const void* __restrict__ w, int w_fp32, int H,
                                                                int8_t* __restrict__ q, bf16* __restrict__ scale) {
  __shared__ float red[8];
  const long long row = blockIdx.x;
  const float* wf = reinterpret_cast<const float*>(w) + row * H;
  const bf16* wb = reinterpret_cast<const bf16*>(w) + row * H;
  float mx = 0.f;
  for (int i = threadIdx.x; i < H; i += 256) mx = fmaxf(mx, fabsf(w_fp32 ? wf[i] : __bfloat162float(wb[i])));
  mx = block_reduce_256<true>(mx, red);
  const float s = fmaxf(mx / 127.f, 1e-12f);
  for (int i = threadIdx.x; i < H; i += 256) {
    const float v = rintf((w_fp32 ? wf[i] : __bfloat162float(wb[i])) / s);
    q[row * H + i] = (int8_t)fminf(fmaxf(v, -127.f), 127.f);
  }
  if (threadIdx.x == 0) scale[row] = __float2bfloat16_rn(s);
}

static int grid_for(long long work) {
  return (int)std::max<long long>(1, std::min<long long>((work + 255) / 256, 148LL * 16));
}

int set_counts(int* p, int nchunks, int step, long long total, cudaStream_t s) {
  set_counts_kernel<<<1, 256, 0, s>>>(p, nchunks, step, total);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

int ce_init(const CeState& st, long long n, int H, cudaStream_t s) {
  if (n == 0) return kOk;
  ce_init_kernel<<<grid_for(st.acc ? n * H : n), 256, 0, s>>>(st, n, H);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

int ce_rows(void* lg, int ld, int Vc, long long v0, const long long* tgt, float softcap, bool need_grad,
            const void* wc, int H, const CeState& st, long long n, cudaStream_t s) {
  SMELB_CHECK_ARG(Vc > 0 && ld >= Vc && ld % 8 == 0 && n <= 2147483647LL && ((uintptr_t)lg & 15) == 0, kErrShape,
                  "ce_rows: Vc=%d ld=%d", Vc, ld);
  if (n == 0) return kOk;
  ce_rows_kernel<<<(int)n, 256, 0, s>>>((bf16*)lg, ld, Vc, v0, tgt, softcap, need_grad ? 1 : 0, (const bf16*)wc, H,
                                        st);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

int ce_acc(const float* parts, int nparts, const CeState& st, long long n, int H, cudaStream_t s) {
  SMELB_CHECK_ARG(H % 4 == 0 && ((uintptr_t)parts & 15) == 0 && ((uintptr_t)st.acc & 15) == 0, kErrShape,
                  "ce_acc: H=%d (multiple of 4) and 16-byte aligned arrays required", H);
  if (n == 0) return kOk;
  ce_acc_kernel<<<grid_for(n * H / 4), 256, 0, s>>>(reinterpret_cast<const float4*>(parts), nparts, st, n, H);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

int ce_finish(const CeState& st, long long n, int H, float denom, float* loss_rows, void* gh, cudaStream_t s) {
  if (n == 0) return kOk;
  ce_finish_kernel<<<grid_for(n * H), 256, 0, s>>>(st, n, H, denom, loss_rows, (bf16*)gh);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

int ce_logits_out(const void* lg, int ld, int Vc, long long n, float softcap, float* out, long long ldo,
                  cudaStream_t s) {
  if (n == 0) return kOk;
  ce_logits_out_kernel<<<grid_for(n * Vc), 256, 0, s>>>((const bf16*)lg, ld, Vc, n, softcap, out, ldo);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

int ce_loss_sum(const float* loss_rows, long long n, float denom, float* loss, cudaStream_t s) {
  ce_loss_sum_kernel<<<1, 256, 0, s>>>(loss_rows, n, denom, loss);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

int int8_rows_quantize(const void* w, bool w_fp32, long long rows, int H, void* q, void* scale, cudaStream_t s) {
  SMELB_CHECK_ARG(rows <= 2147483647LL && H > 0, kErrShape, "int8_rows_quantize: rows=%lld H=%d", rows, H);
  if (rows == 0) return kOk;
  int8_rows_quantize_kernel<<<(int)rows, 256, 0, s>>>(w, w_fp32 ? 1 : 0, H, (int8_t*)q, (bf16*)scale);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

int int8_rows_dequant(const void* q, const void* scale, long long rows, int H, void* out, cudaStream_t s,
                      bool out_fp32) {
  if (rows == 0) return kOk;
  if (out_fp32)
    int8_rows_dequant_kernel<float><<<grid_for(rows * H), 256, 0, s>>>((const int8_t*)q, (const bf16*)scale, rows, H,
                                                                       (float*)out);
  else
    int8_rows_dequant_kernel<bf16><<<grid_for(rows * H), 256, 0, s>>>((const int8_t*)q, (const bf16*)scale, rows, H,
                                                                      (bf16*)out);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

}  // namespace smelb
