// Grouped multi-problem GEMM engine for the MoE expert layer (sm_100a: TMA + tcgen05 + TMEM).
//
// Every GEMM of the layer is expressed "swap-AB": the weight side is the MMA's A operand (M = 128 output features
// per tile) and the token side is the B operand (N = tokens of one expert, 16..256 per tile). Experts with few
// routed tokens then cost N=16-granular MMAs instead of padding to a 128-row M tile.
//
// One launch runs up to kMaxProblems independent problems (e.g. frozen int4 experts + selected bf16 experts +
// shared expert), scheduled as one persistent tile list over all SMs.
//
// A operand sources (per problem):
//   kAInt4K  : frozen experts, int4 group-64 weights W[e][m][k] (forward). TMA stages the packed nibbles and the
//              (scale, zero) pairs into shared memory; four dequant warps expand them to bf16 in the 128B-swizzled
//              K-major UMMA layout.
//   kAInt4MN : frozen experts, int4 weights used transposed, W[e][k][m] (backward dX). Same staging; the dequant
//              warps write the MN-major UMMA layout.
//   kABf16K  : bf16 weights [m][k] loaded by TMA (selected experts, shared expert, router, LoRA factors).
//   kABf16MN : bf16 weights [k][m] loaded by TMA (their transposes in backward).
// Modes:
//   kTokN : tokens along N. Groups = experts; group g covers token rows offsets[e] .. offsets[e]+counts[e]-1 of the
//           token matrix; output C[row][m]. Optional LoRA K-extension: one extra 64-wide k-block whose A comes from
//           tmAe (per-weight [rows, 64]) and whose B comes from tmBe (per-token [rows, 64]).
//   kTokK : tokens along K (LoRA weight gradients). Output per group: C[g][m][n] = sum_tokens A^T B with fixed N.
// Epilogues: bf16 store, GLU (act(gate) * up; tiles hold 64 gate rows + the matching 64 up rows), DGLU (gated
// MLP backward from saved gate/up), fp32 store.
#pragma once

#include "common.cuh"

namespace smelb {

constexpr int kBM = 128;
constexpr int kBK = 64;
#ifndef SMELB_MAX_BN
#define SMELB_MAX_BN 192
#endif
#ifndef SMELB_STAGES
#define SMELB_STAGES 4
#endif
#ifndef SMELB_QSTAGES
#define SMELB_QSTAGES 3
#endif
constexpr int kMaxBN = SMELB_MAX_BN;     // token tile (MMA N) upper bound
constexpr int kStages = SMELB_STAGES;    // operand ring: a weight tile (16 KB) and a token tile (kMaxBN x 128 B)
constexpr int kQStages = SMELB_QSTAGES;  // packed-int4 staging ring
#ifndef SMELB_QSUB
#define SMELB_QSUB 4
#endif
// k-blocks per int4 staging stage: 4 makes each staged weight row 128 bytes (4 x 32 bytes of nibbles), so a stage
// takes half the TMA row requests that 64-byte rows did for the same bytes; a dequant group owns one or two of a
// stage's k-blocks and releases the stage after its last one.
constexpr int kQSub = SMELB_QSUB;
constexpr int kQRowBytes = kQSub * 32;   // one staged K-major weight row: kQSub k-blocks of 64 nibbles
static_assert(kQRowBytes == 64 || kQRowBytes == 128, "staged rows use the 64- or 128-byte swizzle");
constexpr int kMaxProblems = 12;
constexpr int kMaxGroups = 320;  // groups over all problems of one launch

constexpr int kAStageBytes = kBM * kBK * 2;      // 16 KB bf16 A tile
constexpr int kBStageBytes = kMaxBN * kBK * 2;   // bf16 B tile
// Tensor memory (512 columns x 128 lanes of 32 bit): two fp32 accumulators of kMaxBN columns, then one 32-column
// bf16 weight tile per ring stage for the int4 K-major path (the dequant warps store it, the MMA reads A from it).
constexpr int kTmemAcc = kMaxBN;
constexpr int kTmemA0 = 2 * kMaxBN;
static_assert(kTmemA0 + 4 * 32 <= 512 && kTmemA0 + SMELB_STAGES * 32 <= 512, "tensor memory budget exceeded");
constexpr int kQStageBytes = 128 * kQRowBytes;  // nibbles: 128 rows x kQRowBytes (K-major) or kQSub*64 k-rows x 64 B
constexpr int kSZStageBytes = 2 * kQSub * 64 * 4;  // (scale, zero) pairs: 2 halves x kQSub*64 uint32
// 16-byte chunk c of staged K-major row r sits at chunk c ^ qswz(r) (the TMA 64- or 128-byte swizzle)
__host__ __device__ constexpr int qswz(int r) { return kQRowBytes == 128 ? (r & 7) : ((r >> 1) & 3); }

// warp roles: 0 and 2 TMA producers (token and TMA-sourced weight tiles of alternate k-blocks), 1 MMA, 3 TMA (int4
// staging ring), 4-15 dequant (three
// groups of four warps; group g takes the k-blocks whose ring index is g mod 3), then the epilogue: kEpiSubs warps
// per TMEM lane quarter, which split a tile's accumulator columns between them in 16-column chunks (several warps
// per quarter hide the latency of the per-element conversion and store chains).
// Ring waits: a thread that waits on a barrier round must also be one of the arrivals that the barrier's NEXT round
// of the paired barrier needs (it "gates" the ring), otherwise it can fall two phases behind and its parity wait
// then aliases onto a later phase. So the owning TMA producer (fixed per slot: slot parity) and the owning dequant
// group arrive on "full" in every round they wait on "empty" (the group also for slots whose weight tile comes by
// TMA, the producer also for int4 slots where it loads only the token tile). A dequant group waits
// only for the round before each round it owns, and that round cannot complete without its arrival; a group at
// ring index r has passed r - 3, whose wait saw r - 7 consumed, so its wait for r - 4 cannot alias either (this
// needs kNumDeqGroups <= kStages). Every dequant warp waits on and releases every int4 staging stage once.
#ifndef SMELB_DEQ_GROUPS
#define SMELB_DEQ_GROUPS 3
#endif
constexpr int kNumDeqGroups = SMELB_DEQ_GROUPS;
constexpr int kNumDeqWarps = 4;  // per group
#ifndef SMELB_EPI_SUBS
#define SMELB_EPI_SUBS 3
#endif
constexpr int kEpiSubs = SMELB_EPI_SUBS;
constexpr int kNumEpiWarps = 4 * kEpiSubs;
constexpr int kWarpTmaB = 0, kWarpMma = 1, kWarpTmaA = 2, kWarpTmaQ = 3, kWarpDeq0 = 4;
constexpr int kWarpEpi0 = kWarpDeq0 + kNumDeqGroups * kNumDeqWarps;
constexpr int kThreads = (kWarpEpi0 + kNumEpiWarps) * 32;

enum Mode : int { kTokN = 0, kTokK = 1 };
enum AKind : int { kAInt4K = 0, kAInt4MN = 1, kABf16K = 2, kABf16MN = 3 };
enum Epi : int { kEpiStoreBf16 = 0, kEpiGlu = 1, kEpiDGlu = 2, kEpiStoreF32 = 3 };
enum Act : int { kActSilu = 0, kActGeluTanh = 1 };

struct alignas(64) Problem {
  CUtensorMap tmA;   // bf16 A (weights [rows][k] / [k][m], or tokens [rows][m] in kTokK); unused for int4
  CUtensorMap tmB;   // tokens: kTokN [rows][k] K-major (64-row box); kTokK [rows][n] (MN-major B)
  CUtensorMap tmB32; // kTokN tokens with a 32-row box (token tiles of at most 32 rows)
  CUtensorMap tmB16; // kTokN tokens with a 16-row box (valid when b16 is set)
  CUtensorMap tmAe;  // LoRA extension, weight side [nW * e_wrows][64]
  CUtensorMap tmBe;  // LoRA extension, token side [rows][64]
  CUtensorMap tmQ;   // int4 nibbles (uint8): K-major [nW*rows][K/2], box 128 B x 64 rows;
                     //                      MN-major [nW*K][M/2], box 64 B x 256 rows
  CUtensorMap tmSZ;  // (scale | zero << 16) uint32, transposed [nW*G][rows]: K-major box 64 x 4, MN-major 256 x 1

  int mode, a_kind, epi, act;
  int M;        // output features (valid rows of A)
  int K;        // kTokN reduction length (multiple of 64)
  int N;        // kTokK output columns stored (<= 256); the MMA runs on N rounded up to 64
  int BN;       // kTokN token tile (multiple of 64, <= 256)
  int a_wrows;  // bf16 A, kTokN: tensor-map rows per weight index (K-major: rows of W; MN-major: K)
  int a_x0;     // kTokK: column offset into tmA
  int b_x0;     // kTokK: column offset into tmB
  int has_ext;
  int b16;      // kTokN: tmB16 is set, so a token tile loads exactly the rows the MMA reads (a multiple of 16)
  int e_wrows;  // ext A rows per weight index
  int q_rows;   // int4: rows of the stored matrix per weight index (K-major: M-dim rows; MN-major: K rows)
  int q_groups; // int4: groups per stored row (= stored row length / 64)

  const int* counts;   // tokens per expert id
  const int* offsets;  // first token row per expert id (nullptr: prefix sum of counts in group order)
  const int* gid_of;   // group -> expert id (nullptr: identity)
  const int* widx_of;  // group -> weight index (nullptr: same as expert id)
  int ngroups;

  void* C;            // output
  long long c_sm;     // element stride of C along m
  long long c_sn;     // element stride of C along n (token row for kTokN)
  long long c_gs;     // kTokK: element stride between groups
  const bf16* Hin;    // DGLU: saved (gate | up) pre-activations [rows][2*inter]
  bf16* Hout;         // GLU: optional save of (gate | up) [rows][2*inter]
  long long h_ld;     // row stride of Hin/Hout
  int inter;          // gated-MLP intermediate size (offset of up in h)
  float alpha;        // scale applied to the fp32 accumulator before the store
  int m_pad;          // bf16 [token][feature] stores: features [M, m_pad) are written as zeros (0: none)
  int n_inner;        // kTokN tile order: 0 = the weight (M) tiles of one token tile are consecutive, 1 = the token
                      // tiles of one weight tile are consecutive (a weight tile read once from HBM, then from L2)
};

struct LaunchArgs {
  Problem p[kMaxProblems];
  int nprob;
  int* err;
};

}  // namespace smelb
