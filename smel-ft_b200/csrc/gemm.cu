// Persistent grouped multi-problem GEMM for sm_100a: TMA producer warps, a warp-elected tcgen05.mma issuer with TMEM
// accumulators (double-buffered across tiles), three groups of four int4 dequant warps and a team of epilogue warps.
// See gemm.cuh for the operand conventions and the warp roles.
#include <mutex>

#include "gemm.cuh"
#include "host.h"

namespace smelb {

// ------------------------------------------------------------------------------------------ shared-memory plan
constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kStages * kAStageBytes;
constexpr int kOffQ = kOffB + kStages * kBStageBytes;
constexpr int kOffSZ = kOffQ + kQStages * kQStageBytes;
constexpr int kOffTab = kOffSZ + kQStages * kSZStageBytes;
constexpr int kTabInts = 3 * kMaxGroups + (kMaxGroups + kMaxProblems) + (kMaxProblems + 1) + kMaxProblems;
constexpr int kTileTab = 128;  // decoded tiles of this CTA kept in shared memory (later ones are decoded on the fly)
constexpr int kOffTiles = (kOffTab + kTabInts * 4 + 15) & ~15;
constexpr int kOffBar = kOffTiles + kTileTab * 32;
constexpr int kNumBars = 2 * kStages + 2 * kQStages + 5;
constexpr int kOffTmem = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffTmem + 16;
constexpr int kSmemAlloc = kSmemBytes + 1024;  // slack for 1024-byte alignment of the dynamic buffer
static_assert(kSmemAlloc <= 232448, "shared memory budget exceeded");
static_assert(kThreads <= 1024, "too many threads");

struct alignas(16) TileInfo {
  int p, g, widx, mt, m0, n0, n_valid, nkb;
};
static_assert(sizeof(TileInfo) == 32, "tile table entry");

struct Tables {
  int* gcnt;    // [kMaxGroups] tokens of each group
  int* goff;    // [kMaxGroups] first token row of each group
  int* gw;      // [kMaxGroups] weight index of each group
  int* gpre;    // [kMaxGroups + kMaxProblems] exclusive prefix of token tiles per problem (kTokN)
  int* tstart;  // [kMaxProblems + 1] first global tile of each problem
  int* gbase;   // [kMaxProblems] first group slot of each problem
};

__device__ __forceinline__ int mtiles_of(const Problem& P) {
  if (P.mode == kTokN && P.epi == kEpiGlu) return (P.inter + 63) / 64;
  return (P.M + kBM - 1) / kBM;
}

__device__ __forceinline__ TileInfo decode_tile(const LaunchArgs& args, const Tables& T, int t) {
  TileInfo ti;
  int p = 0;
  while (p + 1 < args.nprob && t >= T.tstart[p + 1]) ++p;
  const Problem& P = args.p[p];
  const int local = t - T.tstart[p];
  const int mtiles = mtiles_of(P);
  const int gb = T.gbase[p];
  ti.p = p;
  if (P.mode == kTokN) {
    const int gp = gb + p;  // gpre holds ngroups + 1 entries per problem
    int ntg;
    if (P.n_inner) {
      const int ntt = T.gpre[gp + P.ngroups];  // token tiles of the problem
      ti.mt = local / ntt;
      ntg = local - ti.mt * ntt;
    } else {
      ntg = local / mtiles;
      ti.mt = local - ntg * mtiles;
    }
    int lo = 0, hi = P.ngroups;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (T.gpre[gp + mid] <= ntg) lo = mid; else hi = mid;
    }
    ti.g = lo;
    const int nt = ntg - T.gpre[gp + lo];
    const int cnt = T.gcnt[gb + lo];
    ti.n0 = T.goff[gb + lo] + nt * P.BN;
    ti.n_valid = min(P.BN, cnt - nt * P.BN);
    ti.m0 = (P.epi == kEpiGlu) ? ti.mt * 64 : ti.mt * kBM;
    ti.nkb = P.K / kBK + (P.has_ext ? 1 : 0);
  } else {
    ti.g = local / mtiles;
    ti.mt = local - ti.g * mtiles;
    ti.n0 = T.goff[gb + ti.g];
    ti.n_valid = P.N;
    ti.m0 = ti.mt * kBM;
    ti.nkb = (T.gcnt[gb + ti.g] + kBK - 1) / kBK;
  }
  ti.widx = T.gw[gb + ti.g];
  return ti;
}

// The i-th tile of this CTA (global tile t = blockIdx.x + i * gridDim.x): decoded once in the prologue for the first
// kTileTab tiles, so the warp roles do not each repeat the search.
__device__ __forceinline__ TileInfo tile_at(const LaunchArgs& args, const Tables& T, const TileInfo* tiles, int i, int t) {
  if (i < kTileTab) return tiles[i];
  return decode_tile(args, T, t);
}

// ------------------------------------------------------------------------------------------ int4 dequant helpers
// dq_fast_ok, dq8_fast, dq8_exact (common.cuh): the int4 -> bf16 expansion shared with the small-token kernels.

// 32 packed bytes (64 values sharing one (scale, zero) pair) -> 32 words of two bf16 in k order. The bytes are two
// 16-byte chunks of a staged row: chunk `c0` and `c0 + 1`, each stored at chunk position c ^ swz.
__device__ __forceinline__ void dq64_fast(const uint8_t* src, int c0, int swz, uint32_t sz, uint32_t (&o)[32]) {
  const uint4 v0 = *reinterpret_cast<const uint4*>(src + ((c0 ^ swz) << 4));
  const uint4 v1 = *reinterpret_cast<const uint4*>(src + (((c0 + 1) ^ swz) << 4));
  const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
  const __nv_bfloat162 s2 = bits_bf162((sz & 0xFFFFu) | (sz << 16));
  const __nv_bfloat162 z2 = bits_bf162((sz >> 16) | (sz & 0xFFFF0000u));
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint4 r = dq8_fast(w[c], s2, z2);
    o[4 * c] = r.x;
    o[4 * c + 1] = r.y;
    o[4 * c + 2] = r.z;
    o[4 * c + 3] = r.w;
  }
}

// The same 64 values through fp32 (groups whose values are not all exact in fp32), out of line: it is rare, and the
// kernel's instruction footprint matters more than its speed.
static __device__ __noinline__ void dq64_exact(const uint8_t* src, int c0, int swz, uint32_t sz, uint32_t* o) {
  const float s = __uint_as_float((sz & 0xFFFFu) << 16);
  const float z = __uint_as_float(sz & 0xFFFF0000u);
#pragma unroll 1
  for (int c = 0; c < 8; ++c) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(src + (((c0 + (c >> 2)) ^ swz) << 4) + (c & 3) * 4);
    const uint4 r = dq8_exact(w, s, z);
    o[4 * c] = r.x;
    o[4 * c + 1] = r.y;
    o[4 * c + 2] = r.z;
    o[4 * c + 3] = r.w;
  }
}

__device__ __forceinline__ void dq64(const uint8_t* src, int c0, int swz, uint32_t sz, uint32_t (&o)[32]) {
  if (dq_fast_ok(sz)) {
    dq64_fast(src, c0, swz, sz, o);
  } else {
    uint32_t oc[32];
    dq64_exact(src, c0, swz, sz, oc);
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = oc[i];
  }
}

// ------------------------------------------------------------------------------------------ epilogue math
// act_fwd / tanh_approx (common.cuh): the activations of the GLU epilogue.

// (act(g), d act / d g) in fp32
__device__ __forceinline__ float2 act_and_grad(float g, int act) {
  if (act == kActSilu) {
    const float sg = __fdividef(1.0f, 1.0f + __expf(-g));
    return make_float2(g * sg, sg * (1.0f + g * (1.0f - sg)));
  }
  const float c = 0.7978845608028654f;
  const float t = tanh_approx(c * (g + 0.044715f * g * g * g));
  return make_float2(0.5f * g * (1.0f + t),
                     0.5f * (1.0f + t) + 0.5f * g * (1.0f - t * t) * c * (1.0f + 3.0f * 0.044715f * g * g));
}

// GLU tiles interleave gate and up in 16-row blocks: A row 32*q + j holds gate feature f0 + 16*q + j for j < 16
// and up feature f0 + 16*q + (j - 16) for j >= 16, so one epilogue warp (32 TMEM lanes) owns both halves of 16
// features. This maps an A row to its row in the natural [64 gate | 64 up] staging order.
__device__ __forceinline__ int glu_stage_row(int r) {
  const int q = r >> 5, j = r & 31;
  return (j < 16) ? (q * 16 + j) : (64 + q * 16 + (j - 16));
}

// ------------------------------------------------------------------------------------------ the kernel
__device__ __forceinline__ bool is_int4(const Problem& P) {
  return P.mode == kTokN && (P.a_kind == kAInt4K || P.a_kind == kAInt4MN);
}

// Group tables of a launch, step 1 (out of line: the prologue's registers stay out of the role loops' allocation):
// thread i reads the i-th group's weight slot, row count and first row (0 where the problem has no offsets).
static __device__ __noinline__ void load_group_tables(const LaunchArgs& args, int* gcnt, int* gw, int* goff) {
  int total_groups = 0;
  for (int p = 0; p < args.nprob; ++p) total_groups += args.p[p].ngroups;
  for (int i = threadIdx.x; i < total_groups; i += blockDim.x) {
    int p = 0, g = i;
    while (g >= args.p[p].ngroups) g -= args.p[p++].ngroups;
    const Problem& P = args.p[p];
    const int e = P.gid_of ? P.gid_of[g] : g;
    gw[i] = P.widx_of ? P.widx_of[g] : e;
    gcnt[i] = P.counts[e];
    goff[i] = P.offsets ? P.offsets[e] : 0;
  }
}

__global__ void __launch_bounds__(kThreads, 1) moe_gemm_kernel(const __grid_constant__ LaunchArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t smem_base = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* err = args.err;

  int* tab = reinterpret_cast<int*>(smem + kOffTab);
  Tables T;
  T.gcnt = tab;
  T.goff = tab + kMaxGroups;
  T.gw = tab + 2 * kMaxGroups;
  T.gpre = tab + 3 * kMaxGroups;
  T.tstart = T.gpre + kMaxGroups + kMaxProblems;
  T.gbase = T.tstart + kMaxProblems + 1;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  // full: the stage's token tile landed (1 arrival + bytes) and its weight tile is ready (TMA bytes + 4 arrivals,
  // or 4 dequant-warp arrivals)
  uint64_t* full = bars;
  uint64_t* empty = full + kStages;         // MMAs reading the stage (weight and token tile) are done
  uint64_t* q_full = empty + kStages;       // packed nibbles + (scale, zero) of a stage's kQSub k-blocks landed
  uint64_t* q_empty = q_full + kQStages;    // every dequant warp is done with the staging stage
  uint64_t* acc_full = q_empty + kQStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* mma_drain = acc_full + 4;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + kOffTmem);
  TileInfo* tiles = reinterpret_cast<TileInfo*>(smem + kOffTiles);

  // ---------------------------------------------------------------- prologue: barriers, TMEM, tile tables
  if (warp == kWarpTmaB) {
    if (lane == 0) {
      for (int s = 0; s < kStages; ++s) {
        mbar_init(&full[s], kNumDeqWarps + 1);  // the owning TMA producer + the owning dequant group
        mbar_init(&empty[s], 1);
      }
      for (int s = 0; s < kQStages; ++s) {
        mbar_init(&q_full[s], 1);
        mbar_init(&q_empty[s], kNumDeqGroups * kNumDeqWarps);
      }
      for (int a = 0; a < 2; ++a) {
        mbar_init(&acc_full[a], 1);
        mbar_init(&acc_empty[a], kNumEpiWarps);
      }
      mbar_init(mma_drain, 1);
      fence_mbar_init();
      for (int p = 0; p < args.nprob; ++p) {
        const Problem& P = args.p[p];
        if (P.a_kind == kAInt4K || P.a_kind == kAInt4MN) {
          tma_prefetch_desc(&P.tmQ);
          tma_prefetch_desc(&P.tmSZ);
        } else {
          tma_prefetch_desc(&P.tmA);
        }
        tma_prefetch_desc(&P.tmB);
        if (P.mode == kTokN) tma_prefetch_desc(&P.tmB32);
        if (P.b16) tma_prefetch_desc(&P.tmB16);
        if (P.has_ext) {
          tma_prefetch_desc(&P.tmAe);
          tma_prefetch_desc(&P.tmBe);
        }
      }
    }
  } else if (warp == kWarpMma) {
    tmem_alloc(s_tmem, 512);
    tmem_relinquish();
  }
  // group tables, step 1: every thread reads one group of the launch (its expert id, weight slot, row count and first
  // row) into shared memory, so the scan below reads no global memory (a warp walking the groups 32 at a time paid
  // a dependent global round trip per 32 groups, ~10 us for a routed launch's 256 groups)
  load_group_tables(args, T.gcnt, T.gw, T.goff);
  __syncthreads();
  // step 2: one warp scans the counts per problem: rows (first rows where no offsets are given) and token tiles
  if (warp == kWarpTmaB) {
    int gbase = 0, total = 0;
    for (int p = 0; p < args.nprob; ++p) {
      const Problem& P = args.p[p];
      if (lane == 0) {
        T.gbase[p] = gbase;
        T.tstart[p] = total;
      }
      int carry_rows = 0, carry_tiles = 0;
      const int gp = gbase + p;
      for (int g0 = 0; g0 < P.ngroups; g0 += 32) {
        const int g = g0 + lane;
        const int cnt = g < P.ngroups ? T.gcnt[gbase + g] : 0;
        const int nt = (P.mode == kTokN) ? (cnt + P.BN - 1) / P.BN : 0;
        int rows_inc = cnt, tiles_inc = nt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int r = __shfl_up_sync(0xffffffffu, rows_inc, o);
          const int tt = __shfl_up_sync(0xffffffffu, tiles_inc, o);
          if (lane >= o) {
            rows_inc += r;
            tiles_inc += tt;
          }
        }
        if (g < P.ngroups) {
          if (!P.offsets) T.goff[gbase + g] = carry_rows + rows_inc - cnt;
          T.gpre[gp + g] = carry_tiles + tiles_inc - nt;
        }
        carry_rows += __shfl_sync(0xffffffffu, rows_inc, 31);
        carry_tiles += __shfl_sync(0xffffffffu, tiles_inc, 31);
      }
      if (lane == 0) T.gpre[gp + P.ngroups] = carry_tiles;
      const int mtiles = mtiles_of(P);
      total += (P.mode == kTokN) ? mtiles * carry_tiles : mtiles * P.ngroups;
      gbase += P.ngroups;
    }
    if (lane == 0) T.tstart[args.nprob] = total;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  const int total_tiles = T.tstart[args.nprob];
  {
    const int mine = total_tiles > (int)blockIdx.x ? (total_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
    for (int i = threadIdx.x; i < min(mine, kTileTab); i += blockDim.x)
      tiles[i] = decode_tile(args, T, (int)blockIdx.x + i * (int)gridDim.x);
  }
  __syncthreads();

  if (warp == kWarpTmaB || warp == kWarpTmaA) {
    // ============================================================================ TMA producers (two warps)
    // Producer `prod` owns the ring slots of parity prod (so it waits on and arrives at every round of its slots):
    // per owned k-block it waits for the slot, then one elected lane arms the slot's `full` barrier with the byte
    // count and issues the token tile and, where the weight tile comes by TMA (bf16 weights, the LoRA extension, the
    // token-side A of kTokK), the weight tile too. Each producer pays one wait and one arrival per two k-blocks.
    // The loops run warp-uniform with elected issue: from a lone lane of a diverged warp the same loop was several
    // times slower (measured).
    static_assert(kStages % 2 == 0, "a producer owns the ring slots of one parity");
    const uint32_t prod = warp == kWarpTmaB ? 0u : 1u;
    uint32_t it = 0;
    bool ok = true;
    for (int t = blockIdx.x, i = 0; t < total_tiles && ok; t += gridDim.x, ++i) {
      const TileInfo ti = tile_at(args, T, tiles, i, t);
      const Problem& P = args.p[ti.p];
      const uint32_t it0 = it;
      it += ti.nkb;
      const bool tokk = P.mode == kTokK;
      const bool glu = P.epi == kEpiGlu;
      const bool int4 = is_int4(P);
      const int a_kind = P.a_kind;
      const int ext_kb = (!tokk && P.has_ext) ? ti.nkb - 1 : -1;
      const CUtensorMap* mB = &P.tmB;
      const CUtensorMap* mB32 = &P.tmB32;
      const CUtensorMap* mB16 = &P.tmB16;
      // with the 16-row map, a token tile loads the rows the MMA reads: 64-row boxes, then 32 and / or 16 rows
      const bool exact = !tokk && P.b16;
      const int b_rows = (ti.n_valid + 15) & ~15;
      const CUtensorMap* mBe = &P.tmBe;
      const CUtensorMap* mAmain = &P.tmA;
      const CUtensorMap* mAext = &P.tmAe;
      const int nb = tokk ? (P.N + 63) / 64 : (ti.n_valid + 63) / 64;
      const int b_x0 = P.b_x0;
      const int r0 = ti.m0, r1 = glu ? P.inter + ti.m0 : ti.m0 + 64;
      const int a_wrows = P.a_wrows, e_wrows = P.e_wrows, a_x0 = P.a_x0;
      for (int kb = (int)((it0 & 1u) != prod); kb < ti.nkb; kb += 2) {
        const uint32_t r = it0 + kb;
        const int s = r % kStages;
        if (!mbar_wait_warp(&empty[s], ((r / kStages) & 1) ^ 1, err, kDevErrWaitEmpty, t, kb)) { ok = false; break; }
        if (elect_one()) {
          uint64_t* f = &full[s];
          uint8_t* sB = smem + kOffB + s * kBStageBytes;
          uint8_t* sA = smem + kOffA + s * kAStageBytes;
          const bool ext = kb == ext_kb;
          const bool a_tma = ext || !int4;  // the weight tile comes by TMA (else the dequant warps fill it)
          const bool b32 = !tokk && !ext && ti.n_valid <= 32;
          const uint32_t b_bytes = (exact && !ext) ? (uint32_t)b_rows * 128u : (b32 ? 4096u : (uint32_t)nb * 8192u);
          mbar_arrive_expect_tx(f, b_bytes + (a_tma ? kAStageBytes : 0));
          // token tile
          if (tokk) {  // B = tokens^T (MN-major)
            const int krow = ti.n0 + kb * kBK;
            for (int i = 0; i < nb; ++i) tma_load_2d(sB + i * 8192, mB, b_x0 + 64 * i, krow, f);
          } else if (exact && !ext) {
            const int n64 = b_rows >> 6, rem = b_rows & 63;
            for (int i = 0; i < n64; ++i) tma_load_2d(sB + i * 8192, mB, kb * kBK, ti.n0 + 64 * i, f);
            if (rem & 32) tma_load_2d(sB + n64 * 8192, mB32, kb * kBK, ti.n0 + 64 * n64, f);
            if (rem & 16) tma_load_2d(sB + n64 * 8192 + (rem & 32) * 128, mB16, kb * kBK, ti.n0 + 64 * n64 + (rem & 32), f);
          } else if (b32) {
            tma_load_2d(sB, mB32, kb * kBK, ti.n0, f);
          } else {
            for (int i = 0; i < nb; ++i)
              tma_load_2d(sB + i * 8192, ext ? mBe : mB, ext ? 0 : kb * kBK, ti.n0 + 64 * i, f);
          }
          // weight tile
          if (a_tma) {
            if (tokk) {  // A = tokens^T (MN-major)
              const int krow = ti.n0 + kb * kBK;
              tma_load_2d(sA, mAmain, a_x0 + ti.m0, krow, f);
              tma_load_2d(sA + 8192, mAmain, a_x0 + ti.m0 + 64, krow, f);
            } else if (ext || a_kind == kABf16K) {
              const CUtensorMap* mA = ext ? mAext : mAmain;
              const int wrow = ti.widx * (ext ? e_wrows : a_wrows);
              const int x = ext ? 0 : kb * kBK;
              if (glu) {
#pragma unroll
                for (int qq = 0; qq < 4; ++qq) {
                  tma_load_2d(sA + qq * 4096, mA, x, wrow + r0 + 16 * qq, f);
                  tma_load_2d(sA + qq * 4096 + 2048, mA, x, wrow + r1 + 16 * qq, f);
                }
              } else {
                tma_load_2d(sA, mA, x, wrow + r0, f);
                tma_load_2d(sA + 8192, mA, x, wrow + r1, f);
              }
            } else {  // kABf16MN
              const int wrow = ti.widx * a_wrows + kb * kBK;
              tma_load_2d(sA, mAmain, ti.m0, wrow, f);
              tma_load_2d(sA + 8192, mAmain, ti.m0 + 64, wrow, f);
            }
          }
        }
        __syncwarp();
      }
    }
    // every copy this warp issued must land before the CTA may exit
    for (uint32_t j = (it > (uint32_t)kStages ? it - kStages : 0u); j < it; ++j)
      if ((j & 1u) == prod)
        if (!mbar_wait_warp(&full[j % kStages], (j / kStages) & 1, err, kDevErrTmaDrain)) break;
  } else if (warp == kWarpTmaQ) {
    // ============================================================================ TMA: int4 staging ring (whole warp)
    uint32_t qi = 0;
    bool ok = true;
    for (int t = blockIdx.x, i = 0; t < total_tiles && ok; t += gridDim.x, ++i) {
      const TileInfo ti = tile_at(args, T, tiles, i, t);
      const Problem& P = args.p[ti.p];
      if (!is_int4(P)) continue;
      const bool glu = P.epi == kEpiGlu;
      const bool kmajor = P.a_kind == kAInt4K;
      const int r0 = ti.m0, r1 = glu ? P.inter + ti.m0 : ti.m0 + 64;
      const int nkq = P.K / kBK;
      const CUtensorMap* mQ = &P.tmQ;
      const CUtensorMap* mSZ = &P.tmSZ;
      const int qrow0 = ti.widx * P.q_rows, grow0 = ti.widx * P.q_groups;
      for (int kq = 0; kq * kQSub < nkq; ++kq, ++qi) {
        const int s = qi % kQStages;
        if (!mbar_wait_warp(&q_empty[s], ((qi / kQStages) & 1) ^ 1, err, kDevErrWaitQEmpty, t, kq)) { ok = false; break; }
        uint8_t* sQ = smem + kOffQ + s * kQStageBytes;
        uint8_t* sSZ = smem + kOffSZ + s * kSZStageBytes;
        uint64_t* fb = &q_full[s];
        if (elect_one()) {
          mbar_arrive_expect_tx(fb, kQStageBytes + kSZStageBytes);
          if (kmajor) {
            tma_load_2d(sQ, mQ, kq * kQRowBytes, qrow0 + r0, fb);
            tma_load_2d(sQ + 64 * kQRowBytes, mQ, kq * kQRowBytes, qrow0 + r1, fb);
            tma_load_2d(sSZ, mSZ, r0, grow0 + kq * kQSub, fb);
            tma_load_2d(sSZ + kSZStageBytes / 2, mSZ, r1, grow0 + kq * kQSub, fb);
          } else {
            tma_load_2d(sQ, mQ, ti.m0 / 2, qrow0 + kq * kQSub * kBK, fb);
            tma_load_2d(sSZ, mSZ, kq * kQSub * kBK, grow0 + ti.m0 / 64, fb);
            tma_load_2d(sSZ + kSZStageBytes / 2, mSZ, kq * kQSub * kBK, grow0 + ti.m0 / 64 + 1, fb);
          }
        }
        __syncwarp();
      }
    }
    for (uint32_t j = (qi > (uint32_t)kQStages ? qi - kQStages : 0u); j < qi; ++j)
      if (!mbar_wait_warp(&q_full[j % kQStages], (j / kQStages) & 1, err, kDevErrTmaDrain)) break;
  } else if (warp == kWarpMma) {
    // ============================================================================ MMA issuer (whole warp)
    // The loop runs warp-uniform and each tcgen05 instruction goes out through one elected lane. Per tile the
    // operand descriptors of ring stage 0 are built once; a stage adds its byte offset to the start-address field
    // (shared-memory addresses >> 4 stay below 2^14, so the field never carries). Per k-block: one wait, one fence,
    // four MMAs and the commit that frees the stage. The LoRA extension (always the tile's last k-block) has its own
    // step after the main loop.
    uint32_t it = 0, acc_it = 0;
    bool ok = true, issued = false;
    const uint32_t tmem_u = __shfl_sync(0xffffffffu, tmem_base, 0);
    const uint64_t descA_k = make_sdesc(smem_base + kOffA, 16, 1024), descA_mn = make_sdesc(smem_base + kOffA, 8192, 1024);
    const uint64_t descB_k = make_sdesc(smem_base + kOffB, 16, 1024), descB_mn = make_sdesc(smem_base + kOffB, 8192, 1024);
    for (int t = blockIdx.x, i = 0; t < total_tiles && ok; t += gridDim.x, ++i) {
      const TileInfo ti = tile_at(args, T, tiles, i, t);
      if (ti.nkb == 0) continue;
      const Problem& P = args.p[ti.p];
      const bool tokk = P.mode == kTokK;
      const bool has_ext = !tokk && P.has_ext;
      const int nmain = has_ext ? ti.nkb - 1 : ti.nkb;
      const bool a_tm = P.mode == kTokN && P.a_kind == kAInt4K;  // weight tile in tensor memory
      const bool a_mn = tokk || P.a_kind == kAInt4MN || P.a_kind == kABf16MN;
      // MN-major B (kTokK) must span whole 64-element swizzle atoms; K-major B needs multiples of 16
      const uint32_t n_mma = tokk ? (uint32_t)((ti.n_valid + 63) & ~63) : (uint32_t)((ti.n_valid + 15) & ~15);
      const uint32_t idesc = make_idesc_bf16(n_mma, (a_tm || !a_mn) ? 0u : 1u, tokk ? 1u : 0u);
      const uint64_t b0 = tokk ? descB_mn : descB_k;
      const uint32_t bstep = tokk ? (2048 >> 4) : (32 >> 4);
      // A: K-major steps 32 B per K=16 inside the swizzle atom, MN-major steps two 8-row k-groups (2048 B)
      const uint64_t a0 = a_mn ? descA_mn : descA_k;
      const uint32_t astep = a_mn ? (2048 >> 4) : (32 >> 4);
      const int acc = acc_it & 1;
      if (!mbar_wait_warp(&acc_empty[acc], ((acc_it >> 1) & 1) ^ 1, err, kDevErrWaitAccEmpty, t)) break;
      tc_fence_after();
      issued = true;  // from here on MMAs may be in flight: drain them before TMEM is released, also on errors
      const uint32_t d_tmem = tmem_u + acc * kTmemAcc;
      if (a_tm) {
        for (int kb = 0; kb < nmain; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait_warp(&full[s], (it / kStages) & 1, err, kDevErrWaitFull, t, kb)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_tmem = tmem_u + kTmemA0 + s * 32;
          const uint64_t bs = b0 + (uint64_t)(s * (kBStageBytes >> 4));
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              umma_f16_ts(d_tmem, a_tmem + kk * 8, bs + (uint64_t)(kk * bstep), idesc, (kb | kk) != 0 ? 1u : 0u);
            umma_commit(&empty[s]);
          }
          __syncwarp();
        }
      } else {
        for (int kb = 0; kb < nmain; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait_warp(&full[s], (it / kStages) & 1, err, kDevErrWaitFull, t, kb)) { ok = false; break; }
          tc_fence_after();
          const uint64_t as = a0 + (uint64_t)(s * (kAStageBytes >> 4));
          const uint64_t bs = b0 + (uint64_t)(s * (kBStageBytes >> 4));
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              umma_f16(d_tmem, as + (uint64_t)(kk * astep), bs + (uint64_t)(kk * bstep), idesc, (kb | kk) != 0 ? 1u : 0u);
            umma_commit(&empty[s]);
          }
          __syncwarp();
        }
      }
      if (!ok) break;
      if (has_ext) {  // both operands K-major from the ring
        const int s = it % kStages;
        if (!mbar_wait_warp(&full[s], (it / kStages) & 1, err, kDevErrWaitFull, t, nmain)) { ok = false; break; }
        tc_fence_after();
        const uint32_t idesc_ext = make_idesc_bf16(n_mma, 0u, 0u);
        const uint64_t as = descA_k + (uint64_t)(s * (kAStageBytes >> 4));
        const uint64_t bs = descB_k + (uint64_t)(s * (kBStageBytes >> 4));
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_f16(d_tmem, as + (uint64_t)(kk * (32 >> 4)), bs + (uint64_t)(kk * (32 >> 4)), idesc_ext,
                     (nmain | kk) != 0 ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        __syncwarp();
        ++it;
      }
      if (elect_one()) umma_commit(&acc_full[acc]);
      __syncwarp();
      ++acc_it;
    }
    if (issued) {  // all MMAs must complete before TMEM is released
      if (elect_one()) umma_commit(mma_drain);
      __syncwarp();
      mbar_wait_warp(mma_drain, 0, err, kDevErrTmaDrain);
    }
  } else if (warp < kWarpEpi0) {
    // ============================================================================ int4 dequant (three groups)
    // Group grp owns the k-blocks whose ring index is grp mod kNumDeqGroups and walks only those. Every dequant warp
    // takes part in every int4 staging stage once, in stage order: it waits for a stage before its first k-block
    // there and releases the stage after its last one (a group owns one or two of a 4-k-block stage's k-blocks); a
    // stage where the group owns no k-block is waited for and released on its own when the walk passes it.
    const int grp = (warp - kWarpDeq0) / kNumDeqWarps;
    const int pt = ((warp - kWarpDeq0) % kNumDeqWarps) * 32 + lane;  // 0..127 within the group
    const int lq = warp & 3;                                         // TMEM lane quarter this warp may access
    const int trow = lq * 32 + lane;                                 // weight-tile row this thread stores to TMEM
    const uint32_t tmem_row = tmem_base + ((uint32_t)(lq * 32) << 16) + kTmemA0;
    static_assert(kNumDeqGroups <= kStages, "a dequant group's empty wait must not alias (see the ring note)");
    static_assert(kQSub == 2 || kQSub == 4, "staged rows of 64 or 128 bytes");
    uint32_t it = 0, qi = 0;
    bool ok = true;
    // take part in staging stage `qstage` without owning a k-block of it
    auto pass_stage = [&](uint32_t qstage, int t, int kb) -> bool {
      const int qs = qstage % kQStages;
      if (!mbar_wait(&q_full[qs], (qstage / kQStages) & 1, err, kDevErrWaitQFull, t, kb)) return false;
      __syncwarp();
      if (elect_one()) mbar_arrive(&q_empty[qs]);
      return true;
    };
    for (int t = blockIdx.x, i = 0; t < total_tiles && ok; t += gridDim.x, ++i) {
      const TileInfo ti = tile_at(args, T, tiles, i, t);
      const Problem& P = args.p[ti.p];
      const int nkb = ti.nkb;
      const uint32_t it0 = it;
      it += nkb;
      // first k-block of this tile owned by the group
      const int kb0 = (int)(((uint32_t)grp + kNumDeqGroups - it0 % kNumDeqGroups) % kNumDeqGroups);
      const int nkq = is_int4(P) ? P.K / kBK : 0;          // int4 k-blocks of the tile (staged nibbles)
      const int nstages = (nkq + kQSub - 1) / kQSub;
      const bool kmajor = P.a_kind == kAInt4K;
      // K-major: weight row trow -> TMEM lane trow, 64 bf16 in columns kTmemA0 + 32 s .. +31; the nibble rows are
      // staged swizzled (16-byte chunk c of row r at chunk c ^ qswz(r)).
      // MN-major: k-row kr, half `half` of the 128 output features -> one 128-byte row of the swizzled smem tile.
      const int sr = P.epi == kEpiGlu ? glu_stage_row(trow) : trow;
      // MN-major: the 8 threads of each quarter-warp take 8 consecutive k-rows (one half of the features), so both
      // their 16-byte reads of the 64B-swizzled nibble rows and their 16-byte writes of the 128B-swizzled tile rows
      // fall in 8 distinct bank groups (with two threads per k-row the writes were 2-way conflicted)
      const int kr = (pt & 7) | ((pt >> 4) << 3), half = (pt >> 3) & 1;
      const int q_off = kmajor ? sr * kQRowBytes : kr * 64;  // + j * 64 * 64 for MN-major
      const int sz_off = (kmajor ? (sr >> 6) : half) * (kQSub * 64) + (kmajor ? (sr & 63) : kr);  // + j * 64
      const int swz = kmajor ? qswz(sr) : ((kr >> 1) & 3);  // k-row j * 64 + kr of the stage: (row >> 1) & 3
      int qdone = 0;   // staging stages of this tile the warp has released
      int qheld = -1;  // the staging stage the warp has waited for and not released yet
      for (int kb = kb0; kb < nkb; kb += kNumDeqGroups) {
        const uint32_t r = it0 + kb;
        const int s = r % kStages;
        const bool q4 = kb < nkq;
        const int kq = kb / kQSub;
        if (q4)
          for (; qdone < kq && ok; ++qdone) ok = pass_stage(qi + qdone, t, kb);
        if (!ok) break;
        if (!mbar_wait(&empty[s], ((r / kStages) & 1) ^ 1, err, kDevErrWaitAEmptyDeq, t, kb)) { ok = false; break; }
        if (q4) {
          const int j = kb % kQSub;
          const uint32_t qstage = qi + kq;
          const int qs = qstage % kQStages;
          if (qheld != kq) {
            if (!mbar_wait(&q_full[qs], (qstage / kQStages) & 1, err, kDevErrWaitQFull, t, kb)) { ok = false; break; }
            qheld = kq;
          }
          const uint8_t* sQ = smem + kOffQ + qs * kQStageBytes + q_off + (kmajor ? 0 : j * 64 * 64);
          const uint32_t sz = reinterpret_cast<const uint32_t*>(smem + kOffSZ + qs * kSZStageBytes)[sz_off + j * 64];
          uint32_t o[32];
          dq64(sQ, kmajor ? 2 * j : 2 * half, swz, sz, o);
          // the stage is released after the group's last k-block in it (a group owns one or two of a stage's k-blocks)
          const int kb_next = kb + kNumDeqGroups;
          if (kb_next >= nkq || kb_next / kQSub != kq) {
            __syncwarp();
            if (elect_one()) mbar_arrive(&q_empty[qs]);
            qdone = kq + 1;
            qheld = -1;
          }
          if (kmajor) {
            tc_fence_after();  // the MMAs that read this TMEM stage completed (empty wait above)
            __syncwarp();      // tcgen05.st is warp-collective
            tmem_st32(tmem_row + s * 32, o);
            tmem_st_wait();
            tc_fence_before();
          } else {
            uint8_t* dst = smem + kOffA + s * kAStageBytes + half * 8192 + (kr >> 3) * 1024 + (kr & 7) * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c)
              *reinterpret_cast<uint4*>(dst + ((c ^ (kr & 7)) << 4)) =
                  make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
            fence_proxy_async_smem();
          }
        }
        __syncwarp();
        if (elect_one()) mbar_arrive(&full[s]);  // also for k-blocks whose weight tile comes by TMA: the owner gates
      }
      for (; qdone < nstages && ok; ++qdone) ok = pass_stage(qi + qdone, t, nkb);
      qi += nstages;
    }
  } else {
    // ============================================================================ epilogue warps
    const int q = warp & 3;                     // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;              // accumulator row (A row) owned by this thread
    const int sub = (warp - kWarpEpi0) >> 2;    // which of the quarter's kEpiSubs warps: takes chunks sub, sub + kEpiSubs, ...
    uint32_t acc_it = 0;
    for (int t = blockIdx.x, i = 0; t < total_tiles; t += gridDim.x, ++i) {
      const TileInfo ti = tile_at(args, T, tiles, i, t);
      const Problem& P = args.p[ti.p];
      if (ti.nkb == 0) {
        // kTokK group without tokens: its gradient block is zero
        if (P.mode == kTokK) {
          const int m = ti.m0 + row;
          if (m < P.M) {
            float* C = reinterpret_cast<float*>(P.C) + (long long)ti.g * P.c_gs;
            for (int n = sub; n < P.N; n += kEpiSubs) C[(long long)m * P.c_sm + (long long)n * P.c_sn] = 0.0f;
          }
        }
        continue;
      }
      const int acc = acc_it & 1;
      if (!mbar_wait(&acc_full[acc], (acc_it >> 1) & 1, err, kDevErrWaitAccFull, t)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + acc * kTmemAcc;
      const int n_valid = ti.n_valid;
      const float alpha = P.alpha;
      const int epi = P.epi, act = P.act;
      // Columns are read from TMEM in chunks of 16 (8 for DGLU) with short unrolled bodies: the kernel's instruction
      // footprint, shared by all warp roles, is what limits the epilogue, not its arithmetic.
      if (epi == kEpiGlu) {
        // lanes 0-15 own gate rows and take even token columns, lanes 16-31 own up rows and take odd ones; both need
        // gate and up of their column (one shuffle across the half-warps)
        const bool is_gate = lane < 16;
        const int f = ti.m0 + q * 16 + (lane & 15);
        const bool fvalid = f < P.inter;
        const long long ldc = P.c_sn, ldh = P.h_ld;
        const int inter = P.inter;
        bf16* cp = reinterpret_cast<bf16*>(P.C) + (long long)ti.n0 * ldc + f;
        bf16* hp = P.Hout ? P.Hout + (long long)ti.n0 * ldh + f : nullptr;
        const int par = is_gate ? 0 : 1;
        for (int c = 16 * sub; c < n_valid; c += 16 * kEpiSubs) {
          uint32_t v[16];
          __syncwarp();
          tmem_ld16(tbase + c, v);
          tmem_ld_wait();
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const float mine_e = __uint_as_float(v[2 * jj]), mine_o = __uint_as_float(v[2 * jj + 1]);
            const float other_e = __shfl_xor_sync(0xffffffffu, mine_e, 16);
            const float other_o = __shfl_xor_sync(0xffffffffu, mine_o, 16);
            const float gacc = is_gate ? mine_e : other_o;
            const float uacc = is_gate ? other_e : mine_o;
            const int n = c + 2 * jj + par;
            if (n < n_valid && fvalid) {
              const float gb = bf16_round(gacc * alpha);
              const float ub = bf16_round(uacc * alpha);
              const float ab = bf16_round(act_fwd(gb, act));
              cp[(long long)n * ldc] = __float2bfloat16_rn(ab * ub);
              if (hp) {
                hp[(long long)n * ldh] = __float2bfloat16_rn(gb);
                hp[(long long)n * ldh + inter] = __float2bfloat16_rn(ub);
              }
            }
          }
        }
      } else if (epi == kEpiDGlu) {
        const int m = ti.m0 + row;
        const bool mvalid = m < P.M;
        const long long ldc = P.c_sn, ldh = P.h_ld;
        const int inter = P.inter;
        bf16* cp = reinterpret_cast<bf16*>(P.C) + (long long)ti.n0 * ldc + m;
        const bf16* hp = P.Hin + (long long)ti.n0 * ldh + m;
        for (int c = 8 * sub; c < n_valid; c += 8 * kEpiSubs) {
          // all of the chunk's saved pre-activations are loaded before any store: interleaved with the stores (which
          // the compiler cannot prove disjoint from them) every column would pay a full memory latency
          bf16 hg[8], hu[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int n = c + j;
            const bool ok = n < n_valid && mvalid;
            hg[j] = ok ? __ldg(hp + (long long)n * ldh) : __float2bfloat16_rn(0.0f);
            hu[j] = ok ? __ldg(hp + (long long)n * ldh + inter) : __float2bfloat16_rn(0.0f);
          }
          uint32_t v[8];
          __syncwarp();
          tmem_ld8(tbase + c, v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int n = c + j;
            if (n < n_valid && mvalid) {
              const float da = bf16_round(__uint_as_float(v[j]) * alpha);
              const float2 ad = act_and_grad(__bfloat162float(hg[j]), act);
              cp[(long long)n * ldc] = __float2bfloat16_rn(da * __bfloat162float(hu[j]) * ad.y);
              cp[(long long)n * ldc + inter] = __float2bfloat16_rn(da * ad.x);
            }
          }
        }
      } else if (epi == kEpiStoreBf16 && P.mode == kTokN && P.c_sm == 1 && (P.M & 1) == 0 && (P.c_sn & 1) == 0 &&
                 (reinterpret_cast<uintptr_t>(P.C) & 3) == 0) {
        // bf16 rows [token][feature] with the features of adjacent lanes adjacent in memory: lane pairs exchange half
        // of their columns (one shuffle per column pair) and each lane stores packed feature pairs as 32-bit words,
        // the even lane for the chunk's first 8 tokens, the odd lane for the last 8.
        const int m = ti.m0 + row;
        const int m0 = m & ~1;
        const bool odd = lane & 1;
        // features [M, m_pad) are stored as zeros (the 64-wide LoRA blocks whose unused columns must read as 0)
        const bool mvalid = m0 < max(P.M, P.m_pad);
        const bool lo_ok = m0 < P.M, hi_ok = m0 + 1 < P.M;
        const long long ldc = P.c_sn;
        uint32_t* cp = reinterpret_cast<uint32_t*>(reinterpret_cast<bf16*>(P.C) + (long long)ti.n0 * ldc + m0);
        const long long ldw = ldc >> 1;  // row pitch in 32-bit words
        for (int c = 16 * sub; c < n_valid; c += 16 * kEpiSubs) {
          uint32_t v[16];
          __syncwarp();
          tmem_ld16(tbase + c, v);
          tmem_ld_wait();
          const int tb = c + (odd ? 8 : 0);  // first token this lane stores
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            // the even lane sends column 8 + j and keeps column j; the odd lane sends column j and keeps 8 + j
            const float mine = __uint_as_float(odd ? v[8 + j] : v[j]);
            const float send = __uint_as_float(odd ? v[j] : v[8 + j]);
            const float other = __shfl_xor_sync(0xffffffffu, send, 1);
            const float lo = odd ? other : mine, hi = odd ? mine : other;  // features m0, m0 + 1
            if (mvalid && tb + j < n_valid)
              cp[(long long)(tb + j) * ldw] =
                  bf162_bits(__floats2bfloat162_rn(lo_ok ? lo * alpha : 0.0f, hi_ok ? hi * alpha : 0.0f));
          }
        }
      } else {
        const int m = ti.m0 + row;
        const bool mvalid = m < max(P.M, P.m_pad);
        const float am = m < P.M ? alpha : 0.0f;  // rows [M, m_pad) are stored as zeros
        const long long ldc = P.c_sn;
        const long long base = ((P.mode == kTokK) ? (long long)ti.g * P.c_gs : (long long)ti.n0 * ldc) +
                               (long long)m * P.c_sm;
        const bool f32 = epi != kEpiStoreBf16;
        for (int c = 16 * sub; c < n_valid; c += 16 * kEpiSubs) {
          uint32_t v[16];
          __syncwarp();
          tmem_ld16(tbase + c, v);
          tmem_ld_wait();
          if (!mvalid) continue;
          const int nn = min(16, n_valid - c);
          if (f32) {
            float* cp = reinterpret_cast<float*>(P.C) + base + (long long)c * ldc;
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (j < nn) cp[(long long)j * ldc] = __uint_as_float(v[j]) * alpha;
          } else {
            bf16* cp = reinterpret_cast<bf16*>(P.C) + base + (long long)c * ldc;
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (j < nn) cp[(long long)j * ldc] = __float2bfloat16_rn(am != 0.0f ? __uint_as_float(v[j]) * am : 0.0f);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (elect_one()) mbar_arrive(&acc_empty[acc]);
      ++acc_it;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// ------------------------------------------------------------------------------------------ host side
// One launch path for every caller: the kernel's shared-memory opt-in once per device, the argument checks, the
// optional CUDA-event timing and the launch count. `err` is the 4-word status area the kernel's bounded waits report
// to (the per-device word, or one the caller owns).
static int launch_gemm_impl(LaunchArgs& args, cudaStream_t stream, int dev, int* err) {
  static std::mutex mu;
  static bool configured[64] = {false};
  SMELB_CHECK_ARG(dev >= 0 && dev < 64, kErrArg, "gemm: device %d out of range", dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!configured[dev]) {
      SMELB_CUDA(cudaFuncSetAttribute(moe_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAlloc));
      configured[dev] = true;
    }
  }
  SMELB_CHECK_ARG(args.nprob >= 1 && args.nprob <= kMaxProblems, kErrArg, "gemm: %d problems in one launch",
                  args.nprob);
  int total_groups = 0;
  for (int p = 0; p < args.nprob; ++p) total_groups += args.p[p].ngroups;
  SMELB_CHECK_ARG(total_groups <= kMaxGroups, kErrShape, "gemm: %d groups in one launch (max %d)", total_groups,
                  kMaxGroups);
  SMELB_CHECK_ARG(err != nullptr, kErrArg, "gemm: no status words");
  args.err = err;
  const bool timed = gemm_timing_enabled();
  if (timed) gemm_timing_begin(stream);
  moe_gemm_kernel<<<num_sms(dev), kThreads, kSmemAlloc, stream>>>(args);
  SMELB_CUDA(cudaGetLastError());
  if (timed) gemm_timing_end(stream);
  count_launch();
  return kOk;
}

int launch_gemm(LaunchArgs& args, cudaStream_t stream) {
  int dev = 0;
  SMELB_CUDA(cudaGetDevice(&dev));
  int* err = device_status(dev);
  SMELB_CHECK_ARG(err != nullptr, kErrCuda, "gemm: no device status word");
  return launch_gemm_impl(args, stream, dev, err);
}

int launch_gemm_status(LaunchArgs& args, cudaStream_t stream, int* err) {
  int dev = 0;
  SMELB_CUDA(cudaGetDevice(&dev));
  return launch_gemm_impl(args, stream, dev, err);
}

}  // namespace smelb
