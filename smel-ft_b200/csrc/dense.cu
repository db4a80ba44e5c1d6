// Small-token dense projections with bf16 weights: the router and shared-gate logits (smel/moe.py:162-167) and the
// shared expert's gate/up + GLU and down projection (smel/moe.py:183-201, shared_mlp without LoRA) when a call has a
// handful of tokens. The GEMM engine walks each 128-row weight tile's K one 64-wide k-block after the other on one
// SM (~0.5 us per k-block, 32 of them at K = 2048), so at one token its two shared-expert launches took ~24 us for
// 6 MB of weights and its router launch ~17 us for 1 MB. Here every warp takes whole output rows: a lane loads 8 consecutive k of every 256 of the row (16-byte pieces, a batch of them in flight
// at once), multiplies them with the T token rows staged once per CTA in shared memory (fp32 FMA, which bounds it
// from about 8 tokens on: it takes up to kDenseGemvMaxT), and the warp sums its lanes. Lane t then writes token t's
// output: bf16(sum), or for the GLU the engine's epilogue g = bf16(sum_g), u = bf16(sum_u), bf16(bf16(act(g)) * u).
// The sums are fp32 in a different order than the engine's, so results can differ from it in the last bf16 bit (and
// a near-tie of the router's bf16 logits can then pick another expert).
#include <mutex>

#include "common.cuh"
#include "host.h"
#include "kernels.h"

namespace smelb {

namespace {

constexpr int kDenseThreads = 128;
constexpr int kDenseBatch = 8;  // 16-byte weight pieces a lane has in flight (a whole 2048-long row)

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 g = __bfloat1622float2(p[j]);
    f[2 * j] = g.x;
    f[2 * j + 1] = g.y;
  }
}

template <bool kGlu>
__global__ void __launch_bounds__(kDenseThreads) dense_gemv_kernel(const DenseGemvArgs a) {
  extern __shared__ uint4 xsm[];  // [T][K / 8]
  const int T = a.T, kv = a.K / 8;
  for (int i = threadIdx.x; i < T * kv; i += blockDim.x) {
    const int t = i / kv, v = i - t * kv;
    xsm[i] = __ldg(reinterpret_cast<const uint4*>(a.x + (long long)t * a.ldx) + v);
  }
  __syncthreads();
  constexpr int NR = kGlu ? 2 : 1;
  const int lane = threadIdx.x & 31;
  const int units = kGlu ? a.inter : a.M + a.M2;
  const long long nw = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long u = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; u < units; u += nw) {
    // the unit's weight row (the second projection's rows follow the first's) and its output column
    const bool second = !kGlu && u >= a.M;
    const long long col = second ? u - a.M : u;
    const bf16* wbase = second ? a.w2 + col * a.ldw2 : a.w + col * a.ldw;
    float acc[NR][kDenseGemvMaxT];
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
      for (int t = 0; t < kDenseGemvMaxT; ++t) acc[r][t] = 0.f;
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      const uint4* wr = reinterpret_cast<const uint4*>(wbase + (long long)r * a.inter * a.ldw);
      for (int v0 = lane; v0 < kv; v0 += 32 * kDenseBatch) {
        uint4 wv[kDenseBatch];
#pragma unroll
        for (int q = 0; q < kDenseBatch; ++q)
          if (v0 + 32 * q < kv) wv[q] = __ldg(wr + v0 + 32 * q);
#pragma unroll
        for (int q = 0; q < kDenseBatch; ++q) {
          if (v0 + 32 * q >= kv) break;
          float wf[8];
          unpack8(wv[q], wf);
#pragma unroll
          for (int t = 0; t < kDenseGemvMaxT; ++t) {
            if (t >= T) break;
            float xf[8];
            unpack8(xsm[t * kv + v0 + 32 * q], xf);
            float s = acc[r][t];
#pragma unroll
            for (int j = 0; j < 8; ++j) s = fmaf(wf[j], xf[j], s);
            acc[r][t] = s;
          }
        }
      }
    }
    // every lane ends with every token's total; lane t keeps token t's
    float mine[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      mine[r] = 0.f;
#pragma unroll
      for (int t = 0; t < kDenseGemvMaxT; ++t) {
        if (t >= T) break;
        float v = acc[r][t];
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == t) mine[r] = v;
      }
    }
    if (lane < T) {
      if (kGlu) {
        const float gb = bf16_round(mine[0]), ub = bf16_round(mine[1]);
        a.out[(long long)lane * a.ldo + u] = __float2bfloat16_rn(bf16_round(act_fwd(gb, a.act)) * ub);
        if (a.hout) {
          a.hout[(long long)lane * a.ldh + u] = __float2bfloat16_rn(gb);
          a.hout[(long long)lane * a.ldh + a.inter + u] = __float2bfloat16_rn(ub);
        }
      } else if (second) {
        a.out2[(long long)lane * a.ldo2 + col] = __float2bfloat16_rn(mine[0]);
      } else {
        a.out[(long long)lane * a.ldo + col] = __float2bfloat16_rn(mine[0]);
      }
    }
  }
}

template <class Kern>
void raise_smem(Kern k, int bytes) {
  static std::mutex mu;
  static int raised[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return;
  std::lock_guard<std::mutex> lk(mu);
  if (raised[dev] < bytes) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess) raised[dev] = bytes;
  }
}

}  // namespace

bool dense_gemv_supported(const DenseGemvArgs& a) {
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return a.T >= 1 && a.T <= kDenseGemvMaxT && a.K >= 8 && a.K % 8 == 0 && a.K <= 4096 && a.ldw % 8 == 0 &&
         a.ldx % 8 == 0 && al16(a.w) && al16(a.x) && (!a.glu || (a.inter >= 1 && 2 * a.inter <= a.M)) &&
         (a.M2 == 0 || (!a.glu && a.M2 > 0 && a.w2 && a.out2 && a.ldw2 % 8 == 0 && al16(a.w2)));
}

int dense_gemv(const DenseGemvArgs& a, cudaStream_t st) {
  SMELB_CHECK_ARG(dense_gemv_supported(a), kErrShape, "dense_gemv: T=%d K=%d", a.T, a.K);
  const int units = a.glu ? a.inter : a.M + a.M2;
  if (units == 0) return kOk;
  const int smem = a.T * a.K * 2;
  const int warps = kDenseThreads / 32;
  int dev = 0;
  SMELB_CUDA(cudaGetDevice(&dev));
  const int blocks = std::min((units + warps - 1) / warps, num_sms(dev) * 4);
  if (a.glu) {
    raise_smem(dense_gemv_kernel<true>, smem);
    dense_gemv_kernel<true><<<blocks, kDenseThreads, smem, st>>>(a);
  } else {
    raise_smem(dense_gemv_kernel<false>, smem);
    dense_gemv_kernel<false><<<blocks, kDenseThreads, smem, st>>>(a);
  }
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

}  // namespace smelb
