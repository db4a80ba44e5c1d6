// Small-token path of the frozen int4 experts (the forward's gate/up + GLU and down projections when each expert
// sees only a few tokens): a dequant-GEMV that streams the packed bank at HBM bandwidth instead of walking 128-row
// weight tiles k-block by k-block through the tcgen05 pipeline on one SM each (smel/moe.py:58-85 with
// smel/quant.py:51-67 fused).
//
// Arithmetic: a group's weights are q s + z (q in 0..15, one (scale, zero) per 64 values of a row), so
//   sum_k (q_k s + z) x_k = s sum_k (128 + q_k) x_k + (z - 128 s) sum_k x_k.
// The tensor core forms sum (128 + q) x with the nibbles taken as bf16 integers 128 + q (one mask per pair: 0x4300
// | q is the bf16 encoding of 128 + q, and every product with a bf16 x is exact in fp32), and sum x as a product with
// A = ones; the group's (scale, zero) are then applied in fp32. Next to the reference, which rounds each dequantized
// weight to bf16 before its product, this differs by that rounding alone (at most 2^-9 of each weight): it takes
// one masking instruction per two weights where the rounded form takes four, and the expansion is what bounds this
// kernel's issue rate.
//
// Work: a task is (active expert, MT output columns). One CTA per SM holds a ring of shared-memory stages, each one
// task's weight rows brought by TMA: the packed nibbles of the tile's full K as boxes of W bytes x MT rows (W = 128,
// 64 or 32, swizzled over W so that the row reads below are free of bank conflicts) and the tile's (scale, zero)
// words as one [groups][MT] box; a GLU task stages the gate rows and the matching up rows. The CTA's 16 warps are two
// groups of 8 that take alternate tasks of the CTA's contiguous share of the task list; a group refills the stage it
// has finished with its next-but-ring task, so the stream never waits on a separate producer. In a group the warps
// are WM column tiles of 16 x WK k-splits. A lane (g = lane / 4, j = lane % 4) takes, per group of 64, the 8 packed
// bytes [8j, 8j + 8) of rows g and g + 8 of its tile as the A fragments of mma.sync m16n8k16 (bf16 in, fp32
// accumulate: at these token counts the multiply is free next to the HBM stream). Inside a word the values pair as
// (i, i + 4), the pairing the nibble layout gives with one mask per pair; the token side (B fragments, 8 tokens per
// n-tile) is permuted to the same k order and, for an expert with up to 8 rows, kept in registers (with its sums)
// while consecutive tasks keep the expert. The WK partial sums of a tile meet in shared memory behind the group's
// one barrier per pass, after which all 256 threads of the group finish one output each: bf16(acc) for the down
// projection, or for gate/up g = bf16(acc_g), u = bf16(acc_u), a = bf16(bf16(act(g)) * u) (the GEMM engine's GLU
// epilogue), with (g | u) kept in h when asked.
//
// Which experts are active is known only on the device (the plan's counts), so every CTA first compacts the list of
// experts with rows (and their first rows, when no offsets are given) with each task's cost, the number of 16-token
// passes it takes; the CTAs split the task list into runs of equal cost. Every wait is bounded (status words, as the
// GEMM engine), the warps of a group decide together whether to go on, and copies still in flight after a failed
// wait are waited for before the CTA exits.
#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "host.h"
#include "kernels.h"

namespace smelb {

namespace {

constexpr int kGroupWarps = 8;                   // warps of one group
constexpr int kThreads = 2 * kGroupWarps * 32;  // two groups
constexpr int kMaxIds = 512;
constexpr int kMaxStages = 8;
constexpr int kNT = 2;          // n-tiles of a pass over an expert with more than 8 rows (16 tokens)
constexpr int kXRegGroups = 4;  // groups of token values a warp keeps in registers while its expert stays the same
constexpr int kDevErrGemvFull = 15;  // a group waiting for a staged task

struct GemvParams {
  CUtensorMap tmq;   // q as {W bytes, E * rows_w rows, K / 2W chunks}, box {W, MT, K / 2W}, swizzled over W
  CUtensorMap tmsz;  // sz as [E * groups][rows_w] words, box {MT, groups}
  GemvArgs a;
  int part_q, part_sz, stage, nstage;  // part_sz: the (scale, zero) box's stride (128-byte aligned)
  uint32_t bytes;                            // bytes one task's copies bring
  int* err;
};

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// All 256 threads of a group agree on `v` (the AND of every thread's value).
__device__ __forceinline__ bool group_all(int grp, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %2, 0;\n\t"
      "bar.red.and.pred q, %1, 256, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(1 + grp), "r"((uint32_t)v)
      : "memory");
  return r != 0;
}

// One word of 8 nibbles (value i in bits 4i..4i+3) -> 4 bf16 pairs (128 + n_i, 128 + n_{i+4}): 0x4300 | n is the
// bf16 encoding of 128 + n, an integer the tensor core multiplies exactly.
__device__ __forceinline__ void raw_pairs(uint32_t w, uint32_t (&o)[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = ((w >> (4 * i)) & 0x000F000Fu) | 0x43004300u;
}

// A lane's view of a staged part: rows lo = g and hi = g + 8 of its 16-row tile. The 8 bytes [8j, 8j + 8) of group
// ch sit in box ch / (W / 32) at 16-byte chunk (2 (ch mod W / 32) + j / 2), which the TMA swizzle moves to
// chunk ^ (r W / 128 mod W / 16) in row r.
template <int W, int MT>
struct Rows {
  uint32_t lo, hi;  // byte offsets of the rows (+ the half chunk of lane j)
  uint32_t swlo, swhi;
  __device__ __forceinline__ Rows(int rlo, int j) {
    lo = (uint32_t)(rlo * W + (j & 1) * 8);
    hi = (uint32_t)((rlo + 8) * W + (j & 1) * 8);
    swlo = (uint32_t)(((rlo * W) >> 7) & (W / 16 - 1));
    swhi = (uint32_t)((((rlo + 8) * W) >> 7) & (W / 16 - 1));
  }
  __device__ __forceinline__ uint32_t chunk_off(int ch, int j, uint32_t sw) const {
    constexpr int per_box = W / 32;
    const uint32_t c = (uint32_t)((ch % per_box) * 2 + (j >> 1));
    return (uint32_t)((ch / per_box) * MT * W) + ((c ^ sw) << 4);
  }
};

// y += the lane's C fragment of W_group x_group for one group of a staged part: the lane's 8 bytes of rows lo and hi
// at alo / ahi, the rows' (scale, zero) words at zb and zb + 32,
// with W = q s + z folded as s (128 + q) + (z - 128 s): the tensor core sums (128 + q) x in fp32 and the group's
// (scale, zero) apply to that sum and to X = sum of x (in the same C layout: [nt][0] token 2j, [nt][1] 2j + 1).
template <int NT>
__device__ __forceinline__ void group_fold(uint32_t alo, uint32_t ahi, uint32_t zb, const uint32_t (&xp)[NT][2][4],
                                           const float (&X)[NT][2], float (&y)[NT][4]) {
  const uint2 wlo = lds64(alo), whi = lds64(ahi);
  const uint32_t zlo = lds32(zb), zhi = lds32(zb + 32);
  float acc[2][NT][4];  // two chains (word m = 0, 1), summed below
#pragma unroll
  for (int m = 0; m < 2; ++m)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[m][nt][i] = 0.f;
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    uint32_t lo[4], hi[4];
    raw_pairs(m ? wlo.y : wlo.x, lo);
    raw_pairs(m ? whi.y : whi.x, hi);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      mma_16816(acc[m][nt], lo[0], hi[0], lo[1], hi[1], xp[nt][m][0], xp[nt][m][1]);
      mma_16816(acc[m][nt], lo[2], hi[2], lo[3], hi[3], xp[nt][m][2], xp[nt][m][3]);
    }
  }
  const float slo = __uint_as_float(zlo << 16), shi = __uint_as_float(zhi << 16);
  const float zlo_ = fmaf(-128.f, slo, __uint_as_float(zlo & 0xFFFF0000u));
  const float zhi_ = fmaf(-128.f, shi, __uint_as_float(zhi & 0xFFFF0000u));
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    y[nt][0] = fmaf(zlo_, X[nt][0], fmaf(slo, acc[0][nt][0] + acc[1][nt][0], y[nt][0]));
    y[nt][1] = fmaf(zlo_, X[nt][1], fmaf(slo, acc[0][nt][1] + acc[1][nt][1], y[nt][1]));
    y[nt][2] = fmaf(zhi_, X[nt][0], fmaf(shi, acc[0][nt][2] + acc[1][nt][2], y[nt][2]));
    y[nt][3] = fmaf(zhi_, X[nt][1], fmaf(shi, acc[0][nt][3] + acc[1][nt][3], y[nt][3]));
  }
}

// x values [16j, 16j + 16) of group ch for the lane's token of each n-tile (zeros past the expert's rows)
template <int NT>
__device__ __forceinline__ void load_x(const bf16* __restrict__ xs, long long ldx, long long r0, int tok0, int c,
                                       int g, int j, int ch, uint4 (&x)[NT][2]) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int n = tok0 + nt * 8 + g;
    if (n < c) {
      const uint4* p = reinterpret_cast<const uint4*>(xs + (r0 + n) * ldx + ch * 64 + j * 16);
      x[nt][0] = __ldg(p);
      x[nt][1] = __ldg(p + 1);
    } else {
      x[nt][0] = x[nt][1] = make_uint4(0, 0, 0, 0);
    }
  }
}

// The lane's 16 token values of one group as B fragments in the weights' (i, i + 4) pair order (word m of the 16
// values is v[m]; pairs [m][0..3] = (x0, x4), (x1, x5), (x2, x6), (x3, x7) of that word), and the group's sum of x
// per token in the C layout (a product with A = ones).
template <int NT>
__device__ __forceinline__ void pair_x(const uint4 (&v)[NT][2], uint32_t (&xp)[NT][2][4], float (&X)[NT][2]) {
  constexpr uint32_t kOne2 = 0x3F803F80u;  // bf16 (1, 1)
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      xp[nt][m][0] = __byte_perm(v[nt][m].x, v[nt][m].z, 0x5410);
      xp[nt][m][1] = __byte_perm(v[nt][m].x, v[nt][m].z, 0x7632);
      xp[nt][m][2] = __byte_perm(v[nt][m].y, v[nt][m].w, 0x5410);
      xp[nt][m][3] = __byte_perm(v[nt][m].y, v[nt][m].w, 0x7632);
    }
    float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      mma_16816(s, kOne2, kOne2, kOne2, kOne2, xp[nt][m][0], xp[nt][m][1]);
      mma_16816(s, kOne2, kOne2, kOne2, kOne2, xp[nt][m][2], xp[nt][m][3]);
    }
    X[nt][0] = s[0];
    X[nt][1] = s[1];
  }
}

// Partial sums of a pass into red[WK][WM][NACC][NT][4][32] (one of the group's two buffers).
template <int WK, int NACC, int NT>
__device__ __forceinline__ void store_partials(float* red, const float (&acc)[NACC][NT][4], int wm, int wk) {
  constexpr int WM = kGroupWarps / WK;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int u = 0; u < NACC; ++u)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) red[((((wk * WM + wm) * NACC + u) * NT + nt) * 4 + i) * 32 + lane] = acc[u][nt][i];
}

// After the group's barrier, the group's 256 threads finish the pass's outputs: a pair of lanes (l, l ^ 16) of a
// warp takes one output, each summing the WK partials of one accumulator (gate / up; the down projection's lone
// accumulator is split over the WK partials instead), the pair meeting by a shuffle. 16 consecutive outputs are 16
// consecutive columns of one token.
template <bool kGlu, int WK, int NT>
__device__ __forceinline__ void write_outputs(const GemvArgs& a, const float* red, long long r0, int c, int tok0, int m0,
                                              int cols) {
  constexpr int WM = kGroupWarps / WK;
  constexpr int NACC = kGlu ? 2 : 1;
  constexpr int kOut = WM * 16 * 8 * NT;
  const int lane = threadIdx.x & 31, half = lane >> 4;
  const int w = (threadIdx.x & 255) >> 5;
  for (int ob = w * 16; ob < kOut; ob += kGroupWarps * 16) {
    const int o = ob + (lane & 15);
    const int col = o & 15, n_in = (o >> 4) % (8 * NT), om = o / (16 * 8 * NT);
    // fragment element of (col, token): i = 2 (col / 8) + token % 2 in lane 4 (col % 8) + (token % 8) / 2
    const int i = (col >> 3) * 2 + (n_in & 1), ln = (col & 7) * 4 + ((n_in & 7) >> 1), nt = n_in >> 3;
    float v = 0.f;
    if (NACC == 2) {
#pragma unroll
      for (int q = 0; q < WK; ++q) v += red[((((q * WM + om) * NACC + half) * NT + nt) * 4 + i) * 32 + ln];
    } else {
#pragma unroll
      for (int q = half; q < WK; q += 2) v += red[(((q * WM + om) * NT + nt) * 4 + i) * 32 + ln];
    }
    const float other = __shfl_xor_sync(0xffffffffu, v, 16);
    const int n = tok0 + n_in, cg = m0 + om * 16 + col;
    if (half || n >= c || cg >= cols) continue;
    const long long row = r0 + n;
    if (kGlu) {
      const float gb = bf16_round(v), ub = bf16_round(other);
      a.out[row * a.ldo + cg] = __float2bfloat16_rn(bf16_round(act_fwd(gb, a.act)) * ub);
      if (a.hout) {
        a.hout[row * a.ldh + cg] = __float2bfloat16_rn(gb);
        a.hout[row * a.ldh + a.inter + cg] = __float2bfloat16_rn(ub);
      }
    } else {
      a.out[row * a.ldo + cg] = __float2bfloat16_rn(v + other);
    }
  }
}

// Issue the copies of a task (expert e, first column m0) into a stage.
template <int W, int MT, int NACC>
__device__ __forceinline__ void issue_task(const GemvParams& p, uint8_t* st, uint64_t* bar, int e, int m0) {
  const GemvArgs& a = p.a;
  mbar_arrive_expect_tx(bar, p.bytes);
#pragma unroll
  for (int u = 0; u < NACC; ++u) {
    const int row = m0 + u * a.inter;  // gate rows, then the matching up rows
    tma_load_3d(st + u * p.part_q, &p.tmq, 0, e * a.rows_w + row, 0, bar);
    tma_load_2d(st + NACC * p.part_q + u * p.part_sz, &p.tmsz, row, e * (a.K / 64), bar);
  }
}

template <bool kGlu, int WK, int W>
__global__ void __launch_bounds__(kThreads, 1) int4_gemv_kernel(const __grid_constant__ GemvParams p) {
  constexpr int WM = kGroupWarps / WK;
  constexpr int MT = 16 * WM;
  constexpr int NACC = kGlu ? 2 : 1;
  constexpr int kRed = WK * WM * NACC * kNT * 128;  // one buffer of partial sums
  extern __shared__ uint8_t smem_dyn[];
  __shared__ __align__(8) uint64_t full[kMaxStages];
  __shared__ int s_act[kMaxIds], s_off[kMaxIds], s_pass[kMaxIds], s_cnt[kMaxIds];
  __shared__ long long s_cost[kMaxIds + 1];
  __shared__ int s_nact;
  const GemvArgs& a = p.a;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = warp / kGroupWarps, gw = warp % kGroupWarps;  // group, warp in the group
  const int g = lane >> 2, j = lane & 3;
  // stages start at the next 1024-byte boundary (the 128-byte swizzle repeats every 8 rows of 128 bytes)
  const uint32_t st0 = (smem_u32(smem_dyn) + 1023u) & ~1023u;
  uint8_t* const st0p = smem_dyn + (st0 - smem_u32(smem_dyn));
  const int ns = p.nstage;
  const int cols = kGlu ? a.inter : a.rows_w;
  const int tiles = (cols + MT - 1) / MT;
  // after the stages: [group][buffer] partial-sum buffers
  float* const red = reinterpret_cast<float*>(st0p + (size_t)ns * p.stage) + (size_t)grp * 2 * kRed;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  // compact the experts with rows (warp 0, ballot scan in id order) with their first rows (without offsets the
  // experts' rows follow one another in id order: the running sum of the counts before them) and the running cost
  // of their tasks (tiles x 16-token passes)
  if (warp == 0) {
    // every lane's ids, counts and offsets are requested before the scan (one round trip each, not one per 32)
    constexpr int kPer = kMaxIds / 32;
    int ev[kPer], cv[kPer], ov[kPer];
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int i = q * 32 + lane;
      ev[q] = i < a.n_ids ? (a.ids ? a.ids[i] : i) : -1;
    }
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      cv[q] = ev[q] >= 0 ? a.counts[ev[q]] : 0;
      ov[q] = ev[q] >= 0 && a.offsets ? a.offsets[ev[q]] : 0;
    }
    int n = 0, run = 0;
    long long crun = 0;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      if (q * 32 >= a.n_ids) break;
      const int e = ev[q], cnt = cv[q];
      const int pass = (cnt + 15) / 16;
      int incl = cnt;
      long long cincl = (long long)pass * tiles;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        const long long cv2 = __shfl_up_sync(0xffffffffu, cincl, o);
        if (lane >= o) {
          incl += v;
          cincl += cv2;
        }
      }
      const bool on = cnt > 0;
      const unsigned m = __ballot_sync(0xffffffffu, on);
      if (on) {
        const int slot = n + __popc(m & ((1u << lane) - 1));
        s_act[slot] = e;
        s_cnt[slot] = cnt;
        s_off[slot] = a.offsets ? ov[q] : run + incl - cnt;
        s_pass[slot] = pass;
        s_cost[slot] = crun + cincl - (long long)pass * tiles;
      }
      n += __popc(m);
      run += __shfl_sync(0xffffffffu, incl, 31);
      crun += __shfl_sync(0xffffffffu, cincl, 31);
    }
    if (lane == 0) {
      s_nact = n;
      s_cost[n] = crun;
    }
  }
  __syncthreads();
  const int n_act = s_nact;
  // this CTA's run of tasks (expert-major) of equal cost: task t of expert a starts at cost s_cost[a] + (t mod
  // tiles) * s_pass[a]; the run is every task starting in [C b / G, C (b + 1) / G)
  auto first_at = [&](long long pos) -> long long {
    if (pos >= s_cost[n_act]) return (long long)n_act * tiles;
    int lo = 0, hi = n_act - 1;  // the last a with s_cost[a] <= pos
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_cost[mid] <= pos) lo = mid;
      else hi = mid - 1;
    }
    const long long off = pos - s_cost[lo];
    return (long long)lo * tiles + (off + s_pass[lo] - 1) / s_pass[lo];
  };
  const long long C = s_cost[n_act];
  const long long t_beg = first_at(C * blockIdx.x / gridDim.x), t_end = first_at(C * (blockIdx.x + 1) / gridDim.x);
  const int n = (int)(t_end - t_beg);
  const bool leader = (threadIdx.x & 255) == 0;
  const int ai0 = (int)(t_beg / tiles), tile0 = (int)(t_beg - (long long)ai0 * tiles);
  // each group issues its own stages: tasks k = grp, grp + 2, ... use stages k % ns (ns is even)
  if (leader) {
    tma_prefetch_desc(&p.tmq);
    tma_prefetch_desc(&p.tmsz);
    for (int k = grp; k < min(n, ns); k += 2)
      issue_task<W, MT, NACC>(p, st0p + (size_t)k * p.stage, &full[k], s_act[ai0 + (tile0 + k) / tiles],
                              ((tile0 + k) % tiles) * MT);
  }

  const int wm = gw % WM, wk = gw / WM;
  const int groups = a.K / 64;
  const int cpw = (groups + WK - 1) / WK;
  const int ch0 = min(groups, wk * cpw), ch1 = min(groups, ch0 + cpw);
  const bool xreg = ch1 - ch0 <= kXRegGroups;
  const int rlo = wm * 16 + g;  // row lo of the staged part (row hi = rlo + 8)
  const Rows<W, MT> rw(rlo, j);
  // the lane's byte offsets in a staged part for the groups of its k-range kept in registers
  uint32_t xoff_lo[kXRegGroups], xoff_hi[kXRegGroups];
#pragma unroll
  for (int q = 0; q < kXRegGroups; ++q) {
    xoff_lo[q] = rw.lo + rw.chunk_off(ch0 + q, j, rw.swlo);
    xoff_hi[q] = rw.hi + rw.chunk_off(ch0 + q, j, rw.swhi);
  }
  // the warp's token pairs and sums of an expert with up to 8 rows (xreg), kept while the expert stays
  uint32_t xr[kXRegGroups][1][2][4];
  float xX[kXRegGroups][1][2];
  int xr_e = -1, buf = 0;
  int k = grp;
  int ai = ai0 + (tile0 + grp) / tiles, tile = (tile0 + grp) % tiles;  // expert slot and column tile of task k
  for (; k < n; k += 2) {
    const int s = k % ns;
    const int e = s_act[ai];
    const long long r0 = s_off[ai];
    const int c = s_cnt[ai];
    const int m0 = tile * MT;
    const bool live = m0 + wm * 16 < cols;  // warp-uniform
    if (c <= 8 && xreg && e != xr_e) {
      // the token values of this warp's k-range, requested before the stage is waited for
#pragma unroll
      for (int q = 0; q < kXRegGroups; ++q)
        if (ch0 + q < ch1) {
          uint4 v[1][2];
          load_x<1>(a.xs, a.ldx, r0, 0, c, g, j, ch0 + q, v);
          pair_x<1>(v, xr[q], xX[q]);
        }
      xr_e = e;
    }
    const bool ok = mbar_wait(&full[s], (k / ns) & 1, p.err, kDevErrGemvFull, (int)(t_beg + k));
    const uint32_t st = st0 + (uint32_t)(s * p.stage);
    const uint32_t szb = st + (uint32_t)(NACC * p.part_q);
    bool go = true;
    if (c <= 8 && xreg) {
      float acc[NACC][1][4];
#pragma unroll
      for (int u = 0; u < NACC; ++u)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[u][0][i] = 0.f;
      if (live) {
#pragma unroll
        for (int q = 0; q < kXRegGroups; ++q)
          if (ch0 + q < ch1) {
#pragma unroll
            for (int u = 0; u < NACC; ++u)
              group_fold<1>(st + (uint32_t)(u * p.part_q) + xoff_lo[q], st + (uint32_t)(u * p.part_q) + xoff_hi[q],
                            szb + (uint32_t)(u * p.part_sz + (ch0 + q) * MT * 4 + rlo * 4), xr[q], xX[q], acc[u]);
          }
      }
      float* rb = red + buf * kRed;
      store_partials<WK, NACC, 1>(rb, acc, wm, wk);
      go = group_all(grp, ok);  // the stage is consumed and the partials are in place
      if (go) {
        if (leader && k + ns < n)
          issue_task<W, MT, NACC>(p, st0p + (size_t)s * p.stage, &full[s], s_act[ai + (tile + ns) / tiles],
                                  ((tile + ns) % tiles) * MT);
        write_outputs<kGlu, WK, 1>(a, rb, r0, c, 0, tile * MT, cols);
      }
      buf ^= 1;
    } else {
      // hotter experts (or long k-ranges): 16-token passes, token values requested one group ahead
      for (int tok0 = 0; tok0 < c && go; tok0 += 8 * kNT) {
        float acc[NACC][kNT][4];
#pragma unroll
        for (int u = 0; u < NACC; ++u)
#pragma unroll
          for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[u][nt][i] = 0.f;
        if (live && ch0 < ch1) {
          uint4 xn[kNT][2];
          load_x<kNT>(a.xs, a.ldx, r0, tok0, c, g, j, ch0, xn);
          for (int ch = ch0; ch < ch1; ++ch) {
            uint32_t xp[kNT][2][4];
            float X[kNT][2];
            pair_x<kNT>(xn, xp, X);
            if (ch + 1 < ch1) load_x<kNT>(a.xs, a.ldx, r0, tok0, c, g, j, ch + 1, xn);
            const uint32_t olo = rw.lo + rw.chunk_off(ch, j, rw.swlo), ohi = rw.hi + rw.chunk_off(ch, j, rw.swhi);
#pragma unroll
            for (int u = 0; u < NACC; ++u)
              group_fold<kNT>(st + (uint32_t)(u * p.part_q) + olo, st + (uint32_t)(u * p.part_q) + ohi,
                              szb + (uint32_t)(u * p.part_sz + ch * MT * 4 + rlo * 4), xp, X, acc[u]);
          }
        }
        float* rb = red + buf * kRed;
        store_partials<WK, NACC, kNT>(rb, acc, wm, wk);
        go = group_all(grp, ok);
        if (go) {
          if (leader && tok0 + 8 * kNT >= c && k + ns < n)
            issue_task<W, MT, NACC>(p, st0p + (size_t)s * p.stage, &full[s], s_act[ai + (tile + ns) / tiles],
                                    ((tile + ns) % tiles) * MT);
          write_outputs<kGlu, WK, kNT>(a, rb, r0, c, tok0, tile * MT, cols);
        }
        buf ^= 1;
      }
    }
    if (!go) break;
    tile += 2;
    while (tile >= tiles) {
      tile -= tiles;
      ++ai;
    }
  }
  // after a failed wait, the copies this group issued and did not consume must land before the CTA may exit
  if (leader)
    for (int kk = k; kk < min(n, k + ns); kk += 2)
      mbar_wait(&full[kk % ns], (kk / ns) & 1, p.err, kDevErrTmaDrain, -1, kk);
}

template <bool kGlu, int WK>
const void* pick_w(int W) {
  if (W == 128) return (const void*)int4_gemv_kernel<kGlu, WK, 128>;
  if (W == 64) return (const void*)int4_gemv_kernel<kGlu, WK, 64>;
  return (const void*)int4_gemv_kernel<kGlu, WK, 32>;
}

template <bool kGlu>
const void* pick(int wk, int W) {
  switch (wk) {
    case 8: return pick_w<kGlu, 8>(W);
    case 4: return pick_w<kGlu, 4>(W);
    case 2: return pick_w<kGlu, 2>(W);
    default: return pick_w<kGlu, 1>(W);
  }
}

// k-splits: about four groups per warp, at most all eight warps of a group
int k_splits(int K) {
  int wk = 1;
  while (wk < kGroupWarps && K / 64 >= 8 * wk) wk *= 2;
  return wk;
}

// Launch shape of one call: kernel, box width, rows per task, stage bytes and count.
struct Shape {
  const void* fn;
  int W, MT, part_q, part_sz, stage, nstage;
  size_t dyn;
};

constexpr int kSmemBudget = 227 * 1024;

bool shape_of(bool glu, int K, Shape& sh) {
  const int rb = K / 2, groups = K / 64;
  if (K <= 0 || K % 64 != 0 || groups > 256) return false;
  sh.W = rb % 128 == 0 ? 128 : rb % 64 == 0 ? 64 : 32;
  if (rb / sh.W > 256) return false;  // chunks of one copy
  const int wk = k_splits(K);
  sh.fn = glu ? pick<true>(wk, sh.W) : pick<false>(wk, sh.W);
  sh.MT = 16 * (kGroupWarps / wk);
  sh.part_q = sh.MT * rb;
  sh.part_sz = (groups * sh.MT * 4 + 127) & ~127;
  sh.stage = ((glu ? 2 : 1) * (sh.part_q + sh.part_sz) + 1023) & ~1023;
  cudaFuncAttributes attr;
  if (cudaFuncGetAttributes(&attr, sh.fn) != cudaSuccess) return false;
  // two groups x two buffers of partial sums: [WK][WM][NACC][kNT][4][32] floats each (WK x WM = the group's warps)
  const int red = 4 * kGroupWarps * (glu ? 2 : 1) * kNT * 128 * 4;
  const int avail = kSmemBudget - (int)attr.sharedSizeBytes - 1024 - red;
  sh.nstage = std::min(kMaxStages, avail / sh.stage) & ~1;  // an even count: each group owns every other stage
  sh.dyn = (size_t)sh.nstage * sh.stage + red + 1024;
  return sh.nstage >= 2;
}

__global__ void split_counts_kernel(const int* __restrict__ counts, int E, int thr, int* __restrict__ hot,
                                    int* __restrict__ cold) {
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < E; e += gridDim.x * blockDim.x) {
    const int c = counts[e];
    hot[e] = c > thr ? c : 0;
    cold[e] = c > thr ? 0 : c;
  }
}

}  // namespace

int split_counts(const int* counts, int E, int thr, int* hot, int* cold, cudaStream_t st) {
  if (E <= 0) return kOk;
  split_counts_kernel<<<(E + 255) / 256, 256, 0, st>>>(counts, E, thr, hot, cold);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

bool int4_gemv_supported(bool glu, int K) {
  Shape sh;
  return shape_of(glu, K, sh);
}

int int4_gemv(const GemvArgs& a, cudaStream_t st) {
  SMELB_CHECK_ARG(a.K % 64 == 0 && a.K > 0, kErrShape, "gemv: K=%d must be a positive multiple of 64", a.K);
  SMELB_CHECK_ARG(!a.glu || (a.inter > 0 && a.inter % 16 == 0 && a.rows_w >= 2 * a.inter), kErrShape,
                  "gemv: inter=%d rows=%d", a.inter, a.rows_w);
  SMELB_CHECK_ARG(a.glu || (a.rows_w > 0 && a.rows_w % 16 == 0), kErrShape, "gemv: rows=%d must be a multiple of 16",
                  a.rows_w);
  SMELB_CHECK_ARG(a.n_ids >= 0 && a.n_ids <= kMaxIds && a.n_experts >= 1, kErrShape,
                  "gemv: %d experts of %d (at most %d)", a.n_ids, a.n_experts, kMaxIds);
  SMELB_CHECK_ARG(a.ldx % 8 == 0 && (reinterpret_cast<uintptr_t>(a.xs) & 15) == 0, kErrShape,
                  "gemv: token rows must be 16-byte aligned");
  if (a.n_ids == 0) return kOk;
  Shape sh;
  SMELB_CHECK_ARG(shape_of(a.glu, a.K, sh), kErrShape, "gemv: K=%d does not fit two shared-memory stages", a.K);
  int dev = 0;
  SMELB_CUDA(cudaGetDevice(&dev));
  {
    // the dynamic shared-memory limit of each kernel is raised once per device
    static std::mutex mu;
    static const void* raised_fn[64][24] = {};
    static size_t raised[64][24] = {};
    std::lock_guard<std::mutex> lk(mu);
    int slot = 0;
    while (slot < 23 && raised_fn[dev & 63][slot] && raised_fn[dev & 63][slot] != sh.fn) ++slot;
    raised_fn[dev & 63][slot] = sh.fn;
    if (raised[dev & 63][slot] < sh.dyn) {
      SMELB_CUDA(cudaFuncSetAttribute(sh.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sh.dyn));
      raised[dev & 63][slot] = sh.dyn;
    }
  }
  GemvParams p;
  memset(&p, 0, sizeof(p));
  const int groups = a.K / 64;
  // the packed rows as W-byte columns x rows x K / 2W chunks: one copy brings a task part as [chunk][row][W bytes]
  const uint64_t qdims[3] = {(uint64_t)sh.W, (uint64_t)a.n_experts * a.rows_w, (uint64_t)(a.K / 2 / sh.W)};
  const uint64_t qstr[2] = {(uint64_t)(a.K / 2), (uint64_t)sh.W};
  const uint32_t qbox[3] = {(uint32_t)sh.W, (uint32_t)sh.MT, (uint32_t)(a.K / 2 / sh.W)};
  int rc = make_tmap_3d(&p.tmq, a.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, qdims, qstr, qbox, sh.W);
  if (rc != kOk) return rc;
  rc = make_tmap_2d(&p.tmsz, a.sz, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, (uint64_t)a.n_experts * groups, a.rows_w,
                    (uint64_t)a.rows_w * 4, sh.MT, groups, 0);
  if (rc != kOk) return rc;
  p.a = a;
  p.part_q = sh.part_q;
  p.part_sz = sh.part_sz;
  p.stage = sh.stage;
  p.nstage = sh.nstage;
  p.bytes = (uint32_t)((a.glu ? 2 : 1) * (sh.part_q + groups * sh.MT * 4));
  p.err = device_status(dev);
  void* params[] = {&p};
  SMELB_CUDA(cudaLaunchKernel(sh.fn, dim3(num_sms(dev)), dim3(kThreads), params, sh.dyn, st));
  count_launch();
  return kOk;
}

}  // namespace smelb
