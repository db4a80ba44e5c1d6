// C ABI of smelb (include/smelb.h): argument checks, GEMM problem construction and the sequencing of the MoE layer's
// forward and backward launches.
#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>

#include "../../include/smelb.h"
#include "common.cuh"
#include "gemm.cuh"
#include "host.h"
#include "kernels.h"

namespace smelb {
const char* last_error();
long long launch_count();
void set_gemm_timing(bool on);
int read_gemm_timing(double* ms, long long* n);
}

using namespace smelb;

namespace {

constexpr int kVersion = 100;  // 0.1.0
constexpr int kW64 = 64;       // column width of the LoRA token-side buffers and extension blocks

// Dispatch-row count at or below which the forward's frozen int4 experts take the dequant-GEMV (gemv.cu) instead of
// the tile engine: few rows per expert make the call a stream of the touched experts' weights.
std::atomic<long long> g_gemv_rows{512};

// The frozen int4 gate/up (glu) or down matrix over expert-grouped rows on the GEMV (rows_est: the expected number
// of rows over all n_ids experts, which sizes the token tile).
int gemv_frozen(bool glu, const void* xs, long long ldx, const int* counts, const int* offsets, const int* ids,
                int n_ids, int n_experts, const void* q, const uint32_t* sz, int rows_w, int K, int inter, int act, long long rows_est,
                void* out, long long ldo, void* hout, long long ldh, cudaStream_t st) {
  GemvArgs g;
  g.xs = (const bf16*)xs;
  g.ldx = ldx;
  g.counts = counts;
  g.offsets = offsets;
  g.ids = ids;
  g.n_ids = n_ids;
  g.n_experts = n_experts;
  g.q = (const uint8_t*)q;
  g.sz = sz;
  g.rows_w = rows_w;
  g.K = K;
  g.inter = inter;
  g.act = act;
  g.glu = glu;
  const long long busy = std::max(1LL, std::min<long long>(n_ids, rows_est));
  g.tok_hint = (int)std::min<long long>(1 << 20, (rows_est + busy - 1) / busy);
  g.out = (bf16*)out;
  g.ldo = ldo;
  g.hout = (bf16*)hout;
  g.ldh = ldh;
  return int4_gemv(g, st);
}

// ---------------------------------------------------------------------------------------------- tensor maps
int tm_bf16(CUtensorMap* m, const void* p, long long rows, long long cols, int box_rows) {
  return make_tmap_2d(m, p, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, cols, cols * 2, 64, box_rows, 128);
}
int tm_q(CUtensorMap* m, const void* q, long long rows, long long cols, bool mn_major) {
  // packed nibbles of a stored matrix [rows][cols]: [rows][cols/2] bytes. K-major tiles stage kQSub k-blocks per
  // row (kQRowBytes, swizzled over the row so the dequant warps' row reads are free of bank conflicts); MN-major
  // tiles stage kQSub k-blocks of 64 k-rows x 64 B, 64-byte swizzled for the same reason.
  return make_tmap_2d(m, q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rows, cols / 2, cols / 2, mn_major ? 64 : kQRowBytes,
                      mn_major ? kQSub * 64 : 64, mn_major ? 64 : kQRowBytes);
}
int tm_sz(CUtensorMap* m, const uint32_t* sz, long long nw_groups, long long rows, bool mn_major) {
  return make_tmap_2d(m, sz, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, nw_groups, rows, rows * 4,
                      mn_major ? kQSub * 64 : 64, mn_major ? 1 : kQSub, 0);
}

#define TRY(x)               \
  do {                       \
    int rc_ = (x);           \
    if (rc_ != kOk) return rc_; \
  } while (0)

struct Builder {
  LaunchArgs args;
  Builder() {
    memset(&args, 0, sizeof(args));
  }
  Problem& add() {
    Problem& P = args.p[args.nprob++];
    memset(&P, 0, sizeof(P));
    P.alpha = 1.0f;
    return P;
  }
  int launch(cudaStream_t st) { return args.nprob ? launch_gemm(args, st) : kOk; }
};

void groups(Problem& P, const int* counts, const int* offsets, const int* gid, const int* widx, int n) {
  P.counts = counts;
  P.offsets = offsets;
  P.gid_of = gid;
  P.widx_of = widx;
  P.ngroups = n;
}

// Int4 stored matrix of the bank: [nw][rows][cols] nibbles with (scale, zero) per 64 columns.
struct Int4Mat {
  const void* q;
  const uint32_t* sz;
  int nw, rows, cols;
};

// kTokN, A = int4 bank used directly (K-major: M = rows, K = cols) or transposed (MN-major: M = cols, K = rows).
int set_a_int4(Problem& P, const Int4Mat& W, bool mn_major) {
  P.a_kind = mn_major ? kAInt4MN : kAInt4K;
  TRY(tm_q(&P.tmQ, W.q, (long long)W.nw * W.rows, W.cols, mn_major));
  TRY(tm_sz(&P.tmSZ, W.sz, (long long)W.nw * (W.cols / 64), W.rows, mn_major));
  P.q_rows = W.rows;
  P.q_groups = W.cols / 64;
  P.M = mn_major ? W.cols : W.rows;
  P.K = mn_major ? W.rows : W.cols;
  return kOk;
}

// kTokN, A = bf16 weights [nw][rows][cols]; K-major uses rows as M, MN-major uses cols as M.
int set_a_bf16(Problem& P, const void* W, int nw, int rows, int cols, bool mn_major, bool glu) {
  P.a_kind = mn_major ? kABf16MN : kABf16K;
  TRY(tm_bf16(&P.tmA, W, (long long)nw * rows, cols, glu ? 16 : 64));
  P.a_wrows = rows;
  P.M = mn_major ? cols : rows;
  P.K = mn_major ? rows : cols;
  return kOk;
}

// LoRA K-extension: weight side [nw][e_rows][64], token side [tok_rows][64]
int set_ext(Problem& P, const void* Wext, int nw, int e_rows, const void* Xext, long long tok_rows, bool glu) {
  P.has_ext = 1;
  TRY(tm_bf16(&P.tmAe, Wext, (long long)nw * e_rows, kW64, glu ? 16 : 64));
  TRY(tm_bf16(&P.tmBe, Xext, tok_rows, kW64, 64));
  P.e_wrows = e_rows;
  return kOk;
}

int set_b_tokens(Problem& P, const void* X, long long rows, int cols, int BN = kMaxBN) {
  P.mode = kTokN;
  P.BN = BN < kMaxBN ? BN : kMaxBN;
  TRY(tm_bf16(&P.tmB32, X, rows, cols, 32));
  TRY(tm_bf16(&P.tmB16, X, rows, cols, 16));
  P.b16 = 1;
  return tm_bf16(&P.tmB, X, rows, cols, 64);
}

void out_bf16(Problem& P, void* C, long long ldc) {
  P.epi = kEpiStoreBf16;
  P.C = C;
  P.c_sn = ldc;
  P.c_sm = 1;
}

// kTokK LoRA gradient: C[g][m][n] = alpha * sum_k A[k][a_x0 + m] * B[k][b_x0 + n] over the tokens of group g.
int set_tokk(Problem& P, const void* Atok, long long rows, int a_cols, int a_x0, int M, const void* Btok, int b_cols,
             int b_x0, int N, float* C, long long c_sm, long long c_sn, long long c_gs, float alpha) {
  P.mode = kTokK;
  P.a_kind = kABf16MN;
  P.epi = kEpiStoreF32;
  TRY(tm_bf16(&P.tmA, Atok, rows, a_cols, 64));
  TRY(tm_bf16(&P.tmB, Btok, rows, b_cols, 64));
  P.a_x0 = a_x0;
  P.b_x0 = b_x0;
  P.M = M;
  P.N = N;  // columns stored; the MMA width is rounded up inside the kernel
  P.C = C;
  P.c_sm = c_sm;
  P.c_sn = c_sn;
  P.c_gs = c_gs;
  P.alpha = alpha;
  return kOk;
}

// ---------------------------------------------------------------------------------------------- LoRA packing
PackBlock blk(const float* src, long long sj, long long sa, long long sb, int a0, int na, int b0, int nb, float s) {
  PackBlock b;
  b.src = src;
  b.sj = sj;
  b.sa = sa;
  b.sb = sb;
  b.a0 = a0;
  b.na = na;
  b.b0 = b0;
  b.nb = nb;
  b.scale = s;
  return b;
}
PackBlock no_blk() { return blk(nullptr, 0, 0, 0, 0, 0, 0, 0, 0.f); }
// appends one output to the batch (launched once for all LoRA operands of a layer call)
int pack(int J, int OA, int OB, PackBlock b0, PackBlock b1, void* out, PackBatch& batch) {
  SMELB_CHECK_ARG(batch.n < kMaxPacks, kErrArg, "LoRA pack batch full");
  PackSpec& s = batch.spec[batch.n];
  s.J = J;
  s.OA = OA;
  s.OB = OB;
  s.blk[0] = b0;
  s.blk[1] = b1;
  batch.out[batch.n++] = out;
  return kOk;
}

// LoRA parameter set of one gated MLP family (J slots; J = 1 for the shared expert)
struct LoraSet {
  int J, r, H, I;
  float s;
  const float *Ag, *Bg, *Au, *Bu, *Ad, *Bd;
};

// forward operands: xa_w [J,2r,H] = [A_gate; A_up]; gu_ext [J,2I,64] = [[s B_gate, 0], [0, s B_up]];
// z_w [J,r,I] = A_down; dn_ext [J,H,64] = [s B_down, 0]
int pack_fwd(const LoraSet& L, void* xa_w, void* gu_ext, void* z_w, void* dn_ext, PackBatch& st) {
  const int r = L.r, H = L.H, I = L.I;
  TRY(pack(L.J, 2 * r, H, blk(L.Ag, (long long)r * H, H, 1, 0, r, 0, H, 1.f),
           blk(L.Au, (long long)r * H, H, 1, r, r, 0, H, 1.f), xa_w, st));
  TRY(pack(L.J, 2 * I, kW64, blk(L.Bg, (long long)I * r, r, 1, 0, I, 0, r, L.s),
           blk(L.Bu, (long long)I * r, r, 1, I, I, r, r, L.s), gu_ext, st));
  TRY(pack(L.J, r, I, blk(L.Ad, (long long)r * I, I, 1, 0, r, 0, I, 1.f), no_blk(), z_w, st));
  TRY(pack(L.J, H, kW64, blk(L.Bd, (long long)H * r, r, 1, 0, H, 0, r, L.s), no_blk(), dn_ext, st));
  return kOk;
}

// backward operands: dz_w [J,r,H] = s B_down^T; da_ext [J,I,64] = [A_down^T, 0];
// dxa_w [J,2r,2I] = [[s B_gate^T, 0], [0, s B_up^T]]; dx_ext [J,H,64] = [A_gate^T, A_up^T, 0]
int pack_bwd(const LoraSet& L, void* dz_w, void* da_ext, void* dxa_w, void* dx_ext, PackBatch& st) {
  const int r = L.r, H = L.H, I = L.I;
  TRY(pack(L.J, r, H, blk(L.Bd, (long long)H * r, 1, r, 0, r, 0, H, L.s), no_blk(), dz_w, st));
  TRY(pack(L.J, I, kW64, blk(L.Ad, (long long)r * I, 1, I, 0, I, 0, r, 1.f), no_blk(), da_ext, st));
  TRY(pack(L.J, 2 * r, 2 * I, blk(L.Bg, (long long)I * r, 1, r, 0, r, 0, I, L.s),
           blk(L.Bu, (long long)I * r, 1, r, r, r, I, I, L.s), dxa_w, st));
  TRY(pack(L.J, H, kW64, blk(L.Ag, (long long)r * H, 1, H, 0, H, 0, r, 1.f),
           blk(L.Au, (long long)r * H, 1, H, 0, H, r, r, 1.f), dx_ext, st));
  return kOk;
}

struct Flags {
  bool router, routed, shared, sgate, save, topv32, sel, sel_lora, sh_lora, fz_bf16, recompute, ext;
};

int check_layer(const smelb_moe_layer& L, Flags& f) {
  f.router = L.flags & SMELB_F_ROUTER;
  f.routed = L.flags & SMELB_F_ROUTED;
  f.shared = L.flags & SMELB_F_SHARED;
  f.sgate = f.shared && (L.flags & SMELB_F_SHARED_GATE);
  f.save = L.flags & SMELB_F_SAVE;
  f.topv32 = L.flags & SMELB_F_TOPV_FP32;
  f.sel = f.routed && L.n_sel > 0;
  f.sel_lora = f.sel && L.r_sel > 0;
  f.sh_lora = f.shared && L.r_sh > 0;
  f.fz_bf16 = L.gu_q == nullptr && L.fz_gu != nullptr;
  f.recompute = L.flags & SMELB_F_RECOMPUTE;
  f.ext = L.flags & SMELB_F_EXT_DISPATCH;
  SMELB_CHECK_ARG(!f.ext || (f.routed && !f.router), kErrArg,
                  "layer: an external dispatch takes the routed experts (and the shared expert), not the router");
  SMELB_CHECK_ARG(L.T >= 0 && L.H > 0 && L.H % 64 == 0, kErrShape, "layer: H=%lld must be a multiple of 64",
                  (long long)L.H);
  SMELB_CHECK_ARG(L.act == SMELB_ACT_SILU || L.act == SMELB_ACT_GELU_TANH, kErrArg, "layer: unknown activation %d",
                  L.act);
  SMELB_CHECK_ARG(L.act_sh == SMELB_ACT_SILU || L.act_sh == SMELB_ACT_GELU_TANH, kErrArg,
                  "layer: unknown shared activation %d", L.act_sh);
  if (f.routed || f.router) {
    SMELB_CHECK_ARG(L.E >= 1 && L.E <= 512 && L.K >= 1 && L.K <= 32 && L.K <= L.E, kErrShape,
                    "layer: E=%lld K=%lld", (long long)L.E, (long long)L.K);
  }
  if (f.routed) {
    SMELB_CHECK_ARG(L.I > 0 && L.I % 64 == 0, kErrShape, "layer: I=%lld must be a multiple of 64", (long long)L.I);
    SMELB_CHECK_ARG(L.n_sel >= 0 && L.n_sel <= L.E, kErrShape, "layer: n_sel=%lld", (long long)L.n_sel);
    SMELB_CHECK_ARG(L.max_rows >= L.T * L.K + L.n_sel * 64, kErrWorkspace, "layer: max_rows=%lld < T*K + 64*n_sel",
                    (long long)L.max_rows);
    SMELB_CHECK_ARG(L.E - L.n_sel + L.n_sel + 2 <= kMaxGroups, kErrShape, "layer: too many experts for one launch");
  }
  if (f.shared) SMELB_CHECK_ARG(L.S > 0 && L.S % 64 == 0, kErrShape, "layer: S=%lld must be a multiple of 64",
                                (long long)L.S);
  if (f.sel_lora) SMELB_CHECK_ARG(2 * L.r_sel <= kW64, kErrShape, "layer: LoRA rank %lld > 32", (long long)L.r_sel);
  if (f.sh_lora) SMELB_CHECK_ARG(2 * L.r_sh <= kW64, kErrShape, "layer: LoRA rank %lld > 32", (long long)L.r_sh);
  // the LoRA weight-gradient GEMMs start TMA boxes at column r of the 64-wide token-side blocks: 16-byte aligned
  // only when r is a multiple of 8
  if (f.sel_lora) SMELB_CHECK_ARG(L.r_sel >= 8 && L.r_sel % 8 == 0, kErrShape,
                                  "layer: LoRA rank %lld (a multiple of 8 is required)", (long long)L.r_sel);
  if (f.sh_lora) SMELB_CHECK_ARG(L.r_sh >= 8 && L.r_sh % 8 == 0, kErrShape,
                                 "layer: shared LoRA rank %lld (a multiple of 8 is required)", (long long)L.r_sh);
  return kOk;
}

// ---------------------------------------------------------------------------------------------- gated-MLP problems
// The gate/up GEMM + GLU epilogue of the shared expert / dense MLP (LoRA as the K-extension): sh_a = act(g) * u, and
// the pre-activations (g | u) into hout when given.
int add_shared_glu(Builder& b, const smelb_moe_layer& L, const Flags& f, void* hout) {
  const int T = (int)L.T, H = (int)L.H, S = (int)L.S;
  Problem& P = b.add();
  TRY(set_a_bf16(P, L.sh_gu, 1, 2 * S, H, false, true));
  TRY(set_b_tokens(P, L.x, T, H));
  groups(P, L.tok_count, nullptr, nullptr, nullptr, 1);
  if (f.sh_lora) TRY(set_ext(P, L.sp_gu_ext, 1, 2 * S, L.sh_xa, T, true));
  P.epi = kEpiGlu;
  P.C = L.sh_a;
  P.c_sn = S;
  P.c_sm = 1;
  P.Hout = (bf16*)hout;
  P.h_ld = 2 * S;
  P.inter = S;
  P.act = L.act_sh;
  return kOk;
}

// The routed gate/up GEMMs + GLU epilogue: frozen experts (int4 bank, or bf16 fz_gu) with row counts fz_counts (left
// out when null) and the selected bf16 experts with their LoRA K-extension, a = act(g) * u over the dispatch rows,
// pre-activations into hout when given.
int add_routed_glu(Builder& b, const smelb_moe_layer& L, const Flags& f, void* hout, const int* fz_counts) {
  const int H = (int)L.H, E = (int)L.E, I = (int)L.I, nsel = (int)L.n_sel, nfz = (int)(L.E - L.n_sel);
  const long long R = L.max_rows;
  if (nfz > 0 && fz_counts) {
    Problem& P = b.add();
    if (f.fz_bf16) TRY(set_a_bf16(P, L.fz_gu, E, 2 * I, H, false, true));
    else TRY(set_a_int4(P, Int4Mat{L.gu_q, L.gu_sz, E, 2 * I, H}, false));
    TRY(set_b_tokens(P, L.xs, R, H));
    groups(P, fz_counts, L.offsets, L.frozen_ids, nullptr, nfz);
    P.epi = kEpiGlu;
    P.C = L.a;
    P.c_sn = I;
    P.c_sm = 1;
    P.Hout = (bf16*)hout;
    P.h_ld = 2 * I;
    P.inter = I;
    P.act = L.act;
  }
  if (f.sel) {
    Problem& P = b.add();
    TRY(set_a_bf16(P, L.sel_gu, nsel, 2 * I, H, false, true));
    TRY(set_b_tokens(P, L.xs, R, H));
    groups(P, L.gcounts, L.offsets, L.sel_ids, L.sel_slots, nsel);
    if (f.sel_lora) TRY(set_ext(P, L.p_gu_ext, nsel, 2 * I, L.xa, R, true));
    P.epi = kEpiGlu;
    P.C = L.a;
    P.c_sn = I;
    P.c_sm = 1;
    P.Hout = (bf16*)hout;
    P.h_ld = 2 * I;
    P.inter = I;
    P.act = L.act;
  }
  return kOk;
}

// Few dispatch rows: the frozen int4 experts stream through the dequant-GEMV (forward, and the backward's recompute
// of the same pre-activations, so that saving and recomputing them give the same bits).
long long routed_rows(const smelb_moe_layer& L, const Flags& f) { return f.ext ? L.max_rows : L.T * L.K; }
bool gemv_fits(int64_t H, int64_t I) { return int4_gemv_supported(true, (int)H) && int4_gemv_supported(false, (int)I); }
bool frozen_on_gemv(const smelb_moe_layer& L, const Flags& f) {
  return f.routed && L.E > L.n_sel && !f.fz_bf16 && routed_rows(L, f) <= g_gemv_rows.load() && gemv_fits(L.H, L.I);
}

// Which frozen experts go where. On the GEMV path with at least kSplitRows dispatch rows (and scratch for the split),
// experts with more than kHotRows rows stay on the tile engine (the GEMV repeats its dequantisation for every 16
// rows, the engine's tensor-core tiles take up to 192 at once) and the rest take the GEMV; a skewed routing at 128
// tokens then costs what it costs on the engine alone, while a call without such experts pays one empty engine
// launch (5-10 us, which is why small calls do not split).
constexpr long long kSplitRows = 1024;
constexpr int kHotRows = 16;
struct FrozenPlan {
  bool gemv, split;
  const int* engine;  // row counts of the frozen experts on the tile engine (null: none there)
  const int* small;   // row counts of the frozen experts on the GEMV
};
FrozenPlan frozen_plan(const smelb_moe_layer& L, const Flags& f) {
  FrozenPlan p;
  p.gemv = frozen_on_gemv(L, f);
  p.split = p.gemv && L.split_counts != nullptr && routed_rows(L, f) >= kSplitRows;
  p.engine = p.gemv ? (p.split ? L.split_counts : nullptr) : L.gcounts;
  p.small = p.split ? L.split_counts + L.E : L.gcounts;
  return p;
}

// The shared expert at a handful of tokens and without LoRA: its gate/up + GLU and its down projection as dense
// GEMVs instead of engine tiles (forward, and the backward's recompute of its pre-activations, so that saving and
// recomputing them agree). Off with the small-token GEMV (smelb_set_gemv_rows(0)).
struct SharedGemv {
  bool on;
  DenseGemvArgs glu, down;
};
// A call with a handful of tokens, with the small-token GEMV switched on (smelb_set_gemv_rows).
bool dense_small(const smelb_moe_layer& L) {
  const long long rows = g_gemv_rows.load();
  return rows > 0 && L.T <= kDenseGemvMaxT && L.T * std::max<long long>(L.K, 1) <= rows;
}
SharedGemv shared_gemv(const smelb_moe_layer& L, const Flags& f, void* hout) {
  SharedGemv g;
  memset(&g, 0, sizeof(g));
  if (!f.shared || f.sh_lora || !dense_small(L)) return g;
  const int T = (int)L.T, H = (int)L.H, S = (int)L.S;
  g.glu = DenseGemvArgs{(const bf16*)L.sh_gu, H, 2 * S, (const bf16*)L.x, H, T, H, true, S, (int)L.act_sh,
                        (bf16*)L.sh_a, S, (bf16*)hout, 2 * S};
  g.down = DenseGemvArgs{(const bf16*)L.sh_dn, S, H, (const bf16*)L.sh_a, S, T, S, false, 0, 0, (bf16*)L.sh_y, H,
                         nullptr, 0};
  g.on = dense_gemv_supported(g.glu) && dense_gemv_supported(g.down);
  return g;
}

// ---------------------------------------------------------------------------------------------- layer forward
int layer_fwd(const smelb_moe_layer& L) {
  Flags f;
  TRY(check_layer(L, f));
  cudaStream_t st = (cudaStream_t)L.stream;
  const int T = (int)L.T, H = (int)L.H, E = (int)L.E, K = (int)L.K, I = (int)L.I, S = (int)L.S;
  const int nsel = (int)L.n_sel, nfz = (int)(L.E - L.n_sel), rs = (int)L.r_sel, rh = (int)L.r_sh;
  const long long R = L.max_rows;
  if (T == 0) return kOk;
  const LoraSet ls{nsel, rs, H, I, L.s_sel, L.A_gate, L.B_gate, L.A_up, L.B_up, L.A_down, L.B_down};
  const LoraSet lh{1, rh, H, S, L.s_sh, L.shA_gate, L.shB_gate, L.shA_up, L.shB_up, L.shA_down, L.shB_down};
  {
    PackBatch pb;
    pb.n = 0;
    if (f.sel_lora) TRY(pack_fwd(ls, L.p_xa_w, L.p_gu_ext, L.p_z_w, L.p_dn_ext, pb));
    if (f.sh_lora) TRY(pack_fwd(lh, L.sp_xa_w, L.sp_gu_ext, L.sp_z_w, L.sp_dn_ext, pb));
    TRY(pack_batch(pb, st));
  }

  // L1: everything that reads only x: router logits, shared gate logit, shared LoRA A product. At a handful of
  // tokens without the shared LoRA the two logit projections are one dense GEMV launch instead.
  DenseGemvArgs lg;
  memset(&lg, 0, sizeof(lg));
  bool logits_dense = false;
  if ((f.router || f.sgate) && !f.sh_lora && dense_small(L)) {
    const bf16* w1 = (const bf16*)(f.router ? L.w_router : L.w_sgate);
    lg = DenseGemvArgs{w1, H, f.router ? E : 1, (const bf16*)L.x, H, T, H, false, 0, 0,
                       (bf16*)(f.router ? L.logits : L.sgate_logit), f.router ? E : 1, nullptr, 0};
    if (f.router && f.sgate) {
      lg.w2 = (const bf16*)L.w_sgate;
      lg.ldw2 = H;
      lg.M2 = 1;
      lg.out2 = (bf16*)L.sgate_logit;
      lg.ldo2 = 1;
    }
    logits_dense = dense_gemv_supported(lg);
  }
  {
    Builder b;
    if (f.router && !logits_dense) {
      Problem& P = b.add();
      TRY(set_a_bf16(P, L.w_router, 1, E, H, false, false));
      TRY(set_b_tokens(P, L.x, T, H));
      groups(P, L.tok_count, nullptr, nullptr, nullptr, 1);
      out_bf16(P, L.logits, E);
    }
    if (f.sgate && !logits_dense) {
      Problem& P = b.add();
      TRY(set_a_bf16(P, L.w_sgate, 1, 1, H, false, false));
      TRY(set_b_tokens(P, L.x, T, H));
      groups(P, L.tok_count, nullptr, nullptr, nullptr, 1);
      out_bf16(P, L.sgate_logit, 1);
    }
    if (f.sh_lora) {
      Problem& P = b.add();
      TRY(set_a_bf16(P, L.sp_xa_w, 1, 2 * rh, H, false, false));
      TRY(set_b_tokens(P, L.x, T, H));
      groups(P, L.tok_count, nullptr, nullptr, nullptr, 1);
      out_bf16(P, L.sh_xa, kW64);
      P.m_pad = kW64;  // the block's unused columns are written as zeros
    }
    TRY(b.launch(st));
    if (logits_dense) TRY(dense_gemv(lg, st));
  }
  if (f.router)
    TRY(router_topk(L.logits, E, T, E, K, L.probs, L.topv, f.topv32, (long long*)L.topi, L.per_expert_scale, st));
  const void* topv = f.router ? L.topv : L.topv_in;
  const long long* topi = (const long long*)(f.router ? L.topi : L.topi_in);

  if (f.routed && !f.ext) {
    // the dispatch buffer xs is written only by the gather that follows, so the plan may use it as scratch
    TRY(dispatch_plan_mt(topi, (long long)T * K, E, L.sel_mask, 64, L.counts, L.gcounts, L.offsets, L.row_of,
                         L.src_of, (long long*)L.order, L.total, (int*)L.xs, (long long)R * H / 2, st));
    TRY(gather_rows(L.x, H, K, L.src_of, L.total, R, L.xs, st));
  }
  const Int4Mat dn{L.dn_q, L.dn_sz, E, H, I};

  // L2: selected-expert LoRA A product, shared expert gate/up (GLU)
  const SharedGemv sg = shared_gemv(L, f, f.save ? L.sh_h : nullptr);
  {
    Builder b;
    if (f.sel_lora) {
      Problem& P = b.add();
      TRY(set_a_bf16(P, L.p_xa_w, nsel, 2 * rs, H, false, false));
      TRY(set_b_tokens(P, L.xs, R, H));
      groups(P, L.gcounts, L.offsets, L.sel_ids, L.sel_slots, nsel);
      out_bf16(P, L.xa, kW64);
      P.m_pad = kW64;  // the block's unused columns are written as zeros
    }
    if (f.shared && !sg.on) TRY(add_shared_glu(b, L, f, f.save ? L.sh_h : nullptr));
    TRY(b.launch(st));
    if (sg.on) TRY(dense_gemv(sg.glu, st));
  }
  const long long rows_est = routed_rows(L, f);
  const FrozenPlan fp = frozen_plan(L, f);
  if (fp.split) TRY(split_counts(L.gcounts, E, kHotRows, L.split_counts, L.split_counts + E, st));
  // L3: routed gate/up (frozen int4 + selected bf16 with LoRA), shared LoRA A of the down projection
  {
    Builder b;
    if (f.routed) TRY(add_routed_glu(b, L, f, f.save ? L.h : nullptr, fp.engine));
    if (f.sh_lora) {
      Problem& P = b.add();
      TRY(set_a_bf16(P, L.sp_z_w, 1, rh, S, false, false));
      TRY(set_b_tokens(P, L.sh_a, T, S));
      groups(P, L.tok_count, nullptr, nullptr, nullptr, 1);
      out_bf16(P, L.sh_z, kW64);
      P.m_pad = kW64;  // the block's unused columns are written as zeros
    }
    TRY(b.launch(st));
  }
  if (fp.gemv)
    TRY(gemv_frozen(true, L.xs, H, fp.small, L.offsets, L.frozen_ids, nfz, E, L.gu_q, L.gu_sz, 2 * I, H, I, L.act,
                    rows_est, L.a, I, f.save ? L.h : nullptr, 2 * I, st));
  // L4: selected LoRA A of the down projection, shared down projection
  {
    Builder b;
    if (f.sel_lora) {
      Problem& P = b.add();
      TRY(set_a_bf16(P, L.p_z_w, nsel, rs, I, false, false));
      TRY(set_b_tokens(P, L.a, R, I));
      groups(P, L.gcounts, L.offsets, L.sel_ids, L.sel_slots, nsel);
      out_bf16(P, L.z, kW64);
      P.m_pad = kW64;  // the block's unused columns are written as zeros
    }
    if (f.shared && !sg.on) {
      Problem& P = b.add();
      TRY(set_a_bf16(P, L.sh_dn, 1, H, S, false, false));
      TRY(set_b_tokens(P, L.sh_a, T, S));
      groups(P, L.tok_count, nullptr, nullptr, nullptr, 1);
      if (f.sh_lora) TRY(set_ext(P, L.sp_dn_ext, 1, H, L.sh_z, T, false));
      out_bf16(P, L.sh_y, H);
    }
    TRY(b.launch(st));
    if (sg.on) TRY(dense_gemv(sg.down, st));
  }
  // L5: routed down projections
  if (fp.gemv)
    TRY(gemv_frozen(false, L.a, I, fp.small, L.offsets, L.frozen_ids, nfz, E, L.dn_q, L.dn_sz, H, I, 0, 0, rows_est,
                    L.y, H, nullptr, 0, st));
  if (f.routed) {
    Builder b;
    if (nfz > 0 && fp.engine) {
      Problem& P = b.add();
      if (f.fz_bf16) TRY(set_a_bf16(P, L.fz_dn, E, H, I, false, false));
      else TRY(set_a_int4(P, dn, false));
      TRY(set_b_tokens(P, L.a, R, I));
      groups(P, fp.engine, L.offsets, L.frozen_ids, nullptr, nfz);
      out_bf16(P, L.y, H);
    }
    if (f.sel) {
      Problem& P = b.add();
      TRY(set_a_bf16(P, L.sel_dn, nsel, H, I, false, false));
      TRY(set_b_tokens(P, L.a, R, I));
      groups(P, L.gcounts, L.offsets, L.sel_ids, L.sel_slots, nsel);
      if (f.sel_lora) TRY(set_ext(P, L.p_dn_ext, nsel, H, L.z, R, false));
      out_bf16(P, L.y, H);
    }
    TRY(b.launch(st));
  }
  if ((f.routed || f.shared) && !f.ext)
    TRY(combine_fwd(f.routed ? L.y : nullptr, L.row_of, topv, f.topv32, T, K, H, f.shared ? L.sh_y : nullptr,
                    f.sgate ? L.sgate_logit : nullptr, L.out, st));
  return kOk;
}

// ---------------------------------------------------------------------------------------------- layer backward
int layer_bwd(const smelb_moe_layer& L) {
  Flags f;
  TRY(check_layer(L, f));
  cudaStream_t st = (cudaStream_t)L.stream;
  const int T = (int)L.T, H = (int)L.H, E = (int)L.E, K = (int)L.K, I = (int)L.I, S = (int)L.S;
  const int nsel = (int)L.n_sel, nfz = (int)(L.E - L.n_sel), rs = (int)L.r_sel, rh = (int)L.r_sh;
  const long long R = L.max_rows;
  const int Epad = (E + 63) / 64 * 64;
  if (T == 0) return kOk;
  const LoraSet ls{nsel, rs, H, I, L.s_sel, L.A_gate, L.B_gate, L.A_up, L.B_up, L.A_down, L.B_down};
  const LoraSet lh{1, rh, H, S, L.s_sh, L.shA_gate, L.shB_gate, L.shA_up, L.shB_up, L.shA_down, L.shB_down};
  {
    PackBatch pb;
    pb.n = 0;
    if (f.sel_lora) TRY(pack_bwd(ls, L.p_dz_w, L.p_da_ext, L.p_dxa_w, L.p_dx_ext, pb));
    if (f.sh_lora) TRY(pack_bwd(lh, L.sp_dz_w, L.sp_da_ext, L.sp_dxa_w, L.sp_dx_ext, pb));
    TRY(pack_batch(pb, st));
  }
  const void* topv = f.router ? L.topv : L.topv_in;

  // R0: without saved gate/up pre-activations (the forward kept only its inputs), recompute them into h / sh_h
  if (f.recompute && (f.routed || f.shared)) {
    SMELB_CHECK_ARG((!f.routed || L.h) && (!f.shared || L.sh_h), kErrArg, "layer_bwd: recompute needs h / sh_h");
    // the forward's split of the frozen experts (its counts are still in split_counts) and the same kernels
    const FrozenPlan fp = frozen_plan(L, f);
    const SharedGemv sg = shared_gemv(L, f, L.sh_h);
    Builder b;
    if (f.shared && !sg.on) TRY(add_shared_glu(b, L, f, L.sh_h));
    if (f.routed) TRY(add_routed_glu(b, L, f, L.h, fp.engine));
    TRY(b.launch(st));
    if (sg.on) TRY(dense_gemv(sg.glu, st));
    if (fp.gemv)
      TRY(gemv_frozen(true, L.xs, H, fp.small, L.offsets, L.frozen_ids, (int)(E - L.n_sel), E, L.gu_q, L.gu_sz, 2 * I,
                      H, I, L.act, routed_rows(L, f), L.a, I, L.h, 2 * I, st));
  }
  if (f.routed && !f.ext)
    TRY(combine_bwd_rows(L.g, L.y, L.src_of, L.total, R, topv, f.topv32, K, H, L.dy, L.dtopv, st));
  const void* sh_dy = L.g;
  if (f.sgate) {
    TRY(shared_gate_bwd(L.g, L.sh_y, L.sgate_logit, T, H, L.sh_dy, L.dgl, st));
    sh_dy = L.sh_dy;
  }
  if (f.router)
    TRY(router_bwd(L.dtopv, f.topv32, L.dprobs, L.probs, (const long long*)L.topi, L.per_expert_scale, T, E, K,
                   L.dlogits, Epad,
                   st));
  const Int4Mat gu{L.gu_q, L.gu_sz, E, 2 * I, H};
  const Int4Mat dn{L.dn_q, L.dn_sz, E, H, I};

  // B1: LoRA products of dy with B_down
  {
    Builder b;
    if (f.sel_lora) {
      Problem& P = b.add();
      TRY(set_a_bf16(P, L.p_dz_w, nsel, rs, H, false, false));
      TRY(set_b_tokens(P, L.dy, R, H));
      groups(P, L.gcounts, L.offsets, L.sel_ids, L.sel_slots, nsel);
      out_bf16(P, L.dz, kW64);
      P.m_pad = kW64;  // the block's unused columns are written as zeros
    }
    if (f.sh_lora) {
      Problem& P = b.add();
      TRY(set_a_bf16(P, L.sp_dz_w, 1, rh, H, false, false));
      TRY(set_b_tokens(P, sh_dy, T, H));
      groups(P, L.tok_count, nullptr, nullptr, nullptr, 1);
      out_bf16(P, L.sh_dz, kW64);
      P.m_pad = kW64;  // the block's unused columns are written as zeros
    }
    TRY(b.launch(st));
  }
  // B2: da = dy @ W_down (+ LoRA) fused with the gated-MLP backward -> dh
  {
    Builder b;
    if (f.routed && nfz > 0) {
      Problem& P = b.add();
      if (f.fz_bf16) TRY(set_a_bf16(P, L.fz_dn, E, H, I, true, false));
      else TRY(set_a_int4(P, dn, true));
      TRY(set_b_tokens(P, L.dy, R, H));
      groups(P, L.gcounts, L.offsets, L.frozen_ids, nullptr, nfz);
      P.epi = kEpiDGlu;
      P.C = L.dh;
      P.c_sn = 2 * I;
      P.Hin = (const bf16*)L.h;
      P.h_ld = 2 * I;
      P.inter = I;
      P.act = L.act;
    }
    if (f.sel) {
      Problem& P = b.add();
      TRY(set_a_bf16(P, L.sel_dn, nsel, H, I, true, false));
      TRY(set_b_tokens(P, L.dy, R, H));
      groups(P, L.gcounts, L.offsets, L.sel_ids, L.sel_slots, nsel);
      if (f.sel_lora) TRY(set_ext(P, L.p_da_ext, nsel, I, L.dz, R, false));
      P.epi = kEpiDGlu;
      P.C = L.dh;
      P.c_sn = 2 * I;
      P.Hin = (const bf16*)L.h;
      P.h_ld = 2 * I;
      P.inter = I;
      P.act = L.act;
    }
    if (f.shared) {
      Problem& P = b.add();
      TRY(set_a_bf16(P, L.sh_dn, 1, H, S, true, false));
      TRY(set_b_tokens(P, sh_dy, T, H));
      groups(P, L.tok_count, nullptr, nullptr, nullptr, 1);
      if (f.sh_lora) TRY(set_ext(P, L.sp_da_ext, 1, S, L.sh_dz, T, false));
      P.epi = kEpiDGlu;
      P.C = L.sh_dh;
      P.c_sn = 2 * S;
      P.Hin = (const bf16*)L.sh_h;
      P.h_ld = 2 * S;
      P.inter = S;
      P.act = L.act_sh;
    }
    TRY(b.launch(st));
  }
  // B3: LoRA products of dh with B_gate / B_up
  {
    Builder b;
    if (f.sel_lora) {
      Problem& P = b.add();
      TRY(set_a_bf16(P, L.p_dxa_w, nsel, 2 * rs, 2 * I, false, false));
      TRY(set_b_tokens(P, L.dh, R, 2 * I));
      groups(P, L.gcounts, L.offsets, L.sel_ids, L.sel_slots, nsel);
      out_bf16(P, L.dxa, kW64);
      P.m_pad = kW64;  // the block's unused columns are written as zeros
    }
    if (f.sh_lora) {
      Problem& P = b.add();
      TRY(set_a_bf16(P, L.sp_dxa_w, 1, 2 * rh, 2 * S, false, false));
      TRY(set_b_tokens(P, L.sh_dh, T, 2 * S));
      groups(P, L.tok_count, nullptr, nullptr, nullptr, 1);
      out_bf16(P, L.sh_dxa, kW64);
      P.m_pad = kW64;  // the block's unused columns are written as zeros
    }
    TRY(b.launch(st));
  }
  // B4: dX contributions: dh @ W_gate_up (+ LoRA) for routed and shared, dlogits @ W_router
  {
    Builder b;
    if (f.routed && nfz > 0) {
      Problem& P = b.add();
      if (f.fz_bf16) TRY(set_a_bf16(P, L.fz_gu, E, 2 * I, H, true, false));
      else TRY(set_a_int4(P, gu, true));
      TRY(set_b_tokens(P, L.dh, R, 2 * I));
      groups(P, L.gcounts, L.offsets, L.frozen_ids, nullptr, nfz);
      out_bf16(P, L.dxs, H);
    }
    if (f.sel) {
      Problem& P = b.add();
      TRY(set_a_bf16(P, L.sel_gu, nsel, 2 * I, H, true, false));
      TRY(set_b_tokens(P, L.dh, R, 2 * I));
      groups(P, L.gcounts, L.offsets, L.sel_ids, L.sel_slots, nsel);
      if (f.sel_lora) TRY(set_ext(P, L.p_dx_ext, nsel, H, L.dxa, R, false));
      out_bf16(P, L.dxs, H);
    }
    if (f.shared) {
      Problem& P = b.add();
      TRY(set_a_bf16(P, L.sh_gu, 1, 2 * S, H, true, false));
      TRY(set_b_tokens(P, L.sh_dh, T, 2 * S));
      groups(P, L.tok_count, nullptr, nullptr, nullptr, 1);
      if (f.sh_lora) TRY(set_ext(P, L.sp_dx_ext, 1, H, L.sh_dxa, T, false));
      out_bf16(P, L.sh_dx, H);
    }
    if (f.router) {
      Problem& P = b.add();
      TRY(set_a_bf16(P, L.w_router, 1, E, H, true, false));
      P.K = Epad;
      TRY(set_b_tokens(P, L.dlogits, T, Epad));
      groups(P, L.tok_count, nullptr, nullptr, nullptr, 1);
      out_bf16(P, L.dx_router, H);
    }
    TRY(b.launch(st));
  }
  // B5: LoRA weight gradients (tokens along K)
  {
    Builder b;
    if (f.sel_lora) {
      const int* gc = L.gcounts;
      auto grp = [&](Problem& P) { groups(P, gc, L.offsets, L.sel_ids, L.sel_slots, nsel); };
      Problem* P;
      P = &b.add();
      TRY(set_tokk(*P, L.xs, R, H, 0, H, L.dxa, kW64, 0, rs, L.gA_gate, 1, H, (long long)rs * H, 1.f));
      grp(*P);
      P = &b.add();
      TRY(set_tokk(*P, L.xs, R, H, 0, H, L.dxa, kW64, rs, rs, L.gA_up, 1, H, (long long)rs * H, 1.f));
      grp(*P);
      P = &b.add();
      TRY(set_tokk(*P, L.dh, R, 2 * I, 0, I, L.xa, kW64, 0, rs, L.gB_gate, rs, 1, (long long)I * rs, L.s_sel));
      grp(*P);
      P = &b.add();
      TRY(set_tokk(*P, L.dh, R, 2 * I, I, I, L.xa, kW64, rs, rs, L.gB_up, rs, 1, (long long)I * rs, L.s_sel));
      grp(*P);
      P = &b.add();
      TRY(set_tokk(*P, L.a, R, I, 0, I, L.dz, kW64, 0, rs, L.gA_down, 1, I, (long long)rs * I, 1.f));
      grp(*P);
      P = &b.add();
      TRY(set_tokk(*P, L.dy, R, H, 0, H, L.z, kW64, 0, rs, L.gB_down, rs, 1, (long long)H * rs, L.s_sel));
      grp(*P);
    }
    if (f.sh_lora) {
      auto grp = [&](Problem& P) { groups(P, L.tok_count, nullptr, nullptr, nullptr, 1); };
      Problem* P;
      P = &b.add();
      TRY(set_tokk(*P, L.x, T, H, 0, H, L.sh_dxa, kW64, 0, rh, L.gshA_gate, 1, H, 0, 1.f));
      grp(*P);
      P = &b.add();
      TRY(set_tokk(*P, L.x, T, H, 0, H, L.sh_dxa, kW64, rh, rh, L.gshA_up, 1, H, 0, 1.f));
      grp(*P);
      P = &b.add();
      TRY(set_tokk(*P, L.sh_dh, T, 2 * S, 0, S, L.sh_xa, kW64, 0, rh, L.gshB_gate, rh, 1, 0, L.s_sh));
      grp(*P);
      P = &b.add();
      TRY(set_tokk(*P, L.sh_dh, T, 2 * S, S, S, L.sh_xa, kW64, rh, rh, L.gshB_up, rh, 1, 0, L.s_sh));
      grp(*P);
      P = &b.add();
      TRY(set_tokk(*P, L.sh_a, T, S, 0, S, L.sh_dz, kW64, 0, rh, L.gshA_down, 1, S, 0, 1.f));
      grp(*P);
      P = &b.add();
      TRY(set_tokk(*P, sh_dy, T, H, 0, H, L.sh_z, kW64, 0, rh, L.gshB_down, rh, 1, 0, L.s_sh));
      grp(*P);
    }
    TRY(b.launch(st));
  }
  if (f.ext) return kOk;  // the caller reduces dxs (dispatch order) itself
  TRY(dx_reduce(f.routed ? L.dxs : nullptr, L.row_of, K, T, H, f.shared ? L.sh_dx : nullptr,
                f.router ? L.dx_router : nullptr, f.sgate ? L.dgl : nullptr, L.w_sgate, L.dx, st));
  return kOk;
}

// ---------------------------------------------------------------------------------------------- frozen experts
// A frozen bank for the stand-alone frozen-experts entry points: the int4 group-64 bank (nibbles + packed
// (scale, zero) pairs) or, when gu_w / dn_w are set, plain bf16 weights gate_up [E, 2I, H] and down [E, H, I]
// (smel/moe.py:18-32 BF16Experts).
struct FrozenBank {
  Int4Mat gu, dn;
  const void* gu_w;
  const void* dn_w;
  int E;
};

// A = the bank's gate_up (gate_up = true) or down matrix, K-major (forward) or MN-major (backward, transposed).
int set_a_frozen_w(Problem& P, const FrozenBank& b, bool gate_up, bool mn_major, int H, int I) {
  if (!b.gu_w) return set_a_int4(P, gate_up ? b.gu : b.dn, mn_major);
  if (gate_up) return set_a_bf16(P, b.gu_w, b.E, 2 * I, H, mn_major, !mn_major);
  return set_a_bf16(P, b.dn_w, b.E, H, I, mn_major, false);
}

int frozen_check(const void* xs, int64_t rows, int64_t H, int64_t I, const int32_t* counts, int64_t E, int act,
                 const char* what) {
  SMELB_CHECK_ARG(counts != nullptr && (rows == 0 || xs != nullptr), kErrArg, "%s: null pointer", what);
  SMELB_CHECK_ARG(rows >= 0 && H > 0 && I > 0 && H % 64 == 0 && I % 64 == 0 && E >= 1 && E <= kMaxGroups, kErrShape,
                  "%s: rows=%lld H=%lld I=%lld E=%lld", what, (long long)rows, (long long)H, (long long)I,
                  (long long)E);
  SMELB_CHECK_ARG(act == SMELB_ACT_SILU || act == SMELB_ACT_GELU_TANH, kErrArg, "%s: unknown activation %d", what,
                  act);
  return kOk;
}

// smel/moe.py:110-126 over expert-grouped rows: a = act(xs W_gate^T) * (xs W_up^T) (GLU epilogue, gate/up
// pre-activations kept in h_save when given), out = a W_down^T. err: status words for the launches (nullptr: the
// per-device word).
int frozen_fwd(const FrozenBank& bank, const void* xs, int64_t rows, int64_t H, int64_t I, const int32_t* counts,
               int64_t E, int act, void* h_save, void* a_buf, void* out, cudaStream_t st, int* err) {
  TRY(frozen_check(xs, rows, H, I, counts, E, act, "frozen_experts_fwd"));
  SMELB_CHECK_ARG(a_buf && out, kErrArg, "frozen_experts_fwd: null output");
  if (rows == 0) return kOk;
  if (!bank.gu_w && rows <= g_gemv_rows.load() && gemv_fits(H, I)) {
    TRY(gemv_frozen(true, xs, H, counts, nullptr, nullptr, (int)E, (int)E, bank.gu.q, bank.gu.sz, (int)(2 * I), (int)H,
                    (int)I, act, rows, a_buf, I, h_save, 2 * I, st));
    return gemv_frozen(false, a_buf, I, counts, nullptr, nullptr, (int)E, (int)E, bank.dn.q, bank.dn.sz, (int)H, (int)I, 0,
                       0, rows, out, H, nullptr, 0, st);
  }
  {
    Builder b;
    Problem& P = b.add();
    TRY(set_a_frozen_w(P, bank, true, false, (int)H, (int)I));
    TRY(set_b_tokens(P, xs, rows, (int)H));
    groups(P, counts, nullptr, nullptr, nullptr, (int)E);
    P.epi = kEpiGlu;
    P.C = a_buf;
    P.c_sn = I;
    P.c_sm = 1;
    P.Hout = (bf16*)h_save;
    P.h_ld = 2 * I;
    P.inter = (int)I;
    P.act = act;
    TRY(err ? launch_gemm_status(b.args, st, err) : b.launch(st));
  }
  {
    Builder b;
    Problem& P = b.add();
    TRY(set_a_frozen_w(P, bank, false, false, (int)H, (int)I));
    TRY(set_b_tokens(P, a_buf, rows, (int)I));
    groups(P, counts, nullptr, nullptr, nullptr, (int)E);
    out_bf16(P, out, H);
    TRY(err ? launch_gemm_status(b.args, st, err) : b.launch(st));
  }
  return kOk;
}

// smel/moe.py:128-143: dx of the frozen experts (no weight gradients). Without the saved pre-activations h, the
// gate/up GEMM is recomputed into h_buf first (the reference's save-xs-only memory contract).
int frozen_bwd(const FrozenBank& bank, const void* xs, const void* dy, int64_t rows, int64_t H, int64_t I,
               const int32_t* counts, int64_t E, int act, const void* h, void* h_buf, void* dh_buf, void* dx,
               cudaStream_t st) {
  TRY(frozen_check(dy, rows, H, I, counts, E, act, "frozen_experts_bwd"));
  SMELB_CHECK_ARG(dh_buf && dx, kErrArg, "frozen_experts_bwd: null output");
  SMELB_CHECK_ARG(h || (xs && h_buf), kErrArg, "frozen_experts_bwd: need the saved h or xs and h_buf to recompute");
  if (rows == 0) return kOk;
  if (!h && !bank.gu_w && rows <= g_gemv_rows.load() && gemv_fits(H, I)) {
    // recompute on the GEMV as the forward did (the GLU output goes to dh_buf, overwritten below)
    TRY(gemv_frozen(true, xs, H, counts, nullptr, nullptr, (int)E, (int)E, bank.gu.q, bank.gu.sz, (int)(2 * I), (int)H,
                    (int)I, act, rows, dh_buf, I, h_buf, 2 * I, st));
    h = h_buf;
  }
  if (!h) {
    // recompute gate/up pre-activations into h_buf (the GLU output goes to dh_buf, overwritten below)
    Builder b;
    Problem& P = b.add();
    TRY(set_a_frozen_w(P, bank, true, false, (int)H, (int)I));
    TRY(set_b_tokens(P, xs, rows, (int)H));
    groups(P, counts, nullptr, nullptr, nullptr, (int)E);
    P.epi = kEpiGlu;
    P.C = dh_buf;
    P.c_sn = I;
    P.c_sm = 1;
    P.Hout = (bf16*)h_buf;
    P.h_ld = 2 * I;
    P.inter = (int)I;
    P.act = act;
    TRY(b.launch(st));
    h = h_buf;
  }
  {
    Builder b;
    Problem& P = b.add();
    TRY(set_a_frozen_w(P, bank, false, true, (int)H, (int)I));
    TRY(set_b_tokens(P, dy, rows, (int)H));
    groups(P, counts, nullptr, nullptr, nullptr, (int)E);
    P.epi = kEpiDGlu;
    P.C = dh_buf;
    P.c_sn = 2 * I;
    P.Hin = (const bf16*)h;
    P.h_ld = 2 * I;
    P.inter = (int)I;
    P.act = act;
    TRY(b.launch(st));
  }
  {
    Builder b;
    Problem& P = b.add();
    TRY(set_a_frozen_w(P, bank, true, true, (int)H, (int)I));
    TRY(set_b_tokens(P, dh_buf, rows, (int)(2 * I)));
    groups(P, counts, nullptr, nullptr, nullptr, (int)E);
    out_bf16(P, dx, H);
    TRY(b.launch(st));
  }
  return kOk;
}

// ---------------------------------------------------------------------------------------------- lora_linear
// smel/lora.py:61-83: y = x w^T + s (x A^T) B^T as one GEMM whose last k-block is the LoRA term (token side x A^T,
// weight side s B, both zero-padded to 64 columns). With two LoRA pairs (lora_gate_up over a stacked [2I, Kd] weight)
// pair b acts on the output rows [b N/2, (b+1) N/2): the token side is [x A_0^T | x A_1^T] and the weight side
// block-diagonal. Backward: dz = dy (s B) (same block structure), dx = dy w + dz [A_0; A_1] (one GEMM with the LoRA
// term as its K-extension), dA_b = dz_b^T x and dB_b = s dy_b^T (x A_b^T) as token-reduction GEMMs.
struct LinLayout {
  size_t xa_w, ext, tok, dz, dz_w, dx_ext, total;
};

size_t lin_align(size_t x) { return (x + 255) & ~size_t(255); }

LinLayout lin_layout(int64_t T, int64_t Kd, int64_t N) {
  LinLayout L{};
  size_t o = 0;
  L.tok = o;    o += 256;
  L.xa_w = o;   o += lin_align((size_t)kW64 * Kd * 2);
  L.ext = o;    o += lin_align((size_t)N * kW64 * 2);
  L.dz = o;     o += lin_align((size_t)T * kW64 * 2);
  L.dz_w = o;   o += lin_align((size_t)kW64 * N * 2);
  L.dx_ext = o; o += lin_align((size_t)Kd * kW64 * 2);
  L.total = o;
  return L;
}

struct LinArgs {
  const void* x;
  int64_t T, Kd, N, r;
  const void* w;
  const float *A[2], *B[2];
  int nblk;  // LoRA pairs: 0 (plain GEMM), 1 or 2
  float s;
};

int lin_check(const LinArgs& a, void* ws, int64_t ws_bytes, const char* what) {
  SMELB_CHECK_ARG(a.w && ws && (a.T == 0 || a.x), kErrArg, "%s: null pointer", what);
  SMELB_CHECK_ARG(a.T >= 0 && a.T < (1LL << 31) && a.Kd > 0 && a.Kd % 64 == 0 && a.N > 0 && a.N % 64 == 0 &&
                      a.Kd < (1 << 24) && a.N < (1 << 24),
                  kErrShape, "%s: T=%lld in=%lld out=%lld (in and out must be multiples of 64)", what, (long long)a.T,
                  (long long)a.Kd, (long long)a.N);
  if (a.nblk) {
    // the pairs' columns of the 64-wide token-side block start at multiples of r elements, and a TMA box must start
    // on a 16-byte boundary: r a multiple of 8
    SMELB_CHECK_ARG(a.r >= 8 && a.r % 8 == 0 && a.nblk * a.r <= kW64, kErrShape,
                    "%s: LoRA rank %lld (a multiple of 8, at most %d per pair)", what, (long long)a.r, kW64 / a.nblk);
    SMELB_CHECK_ARG(a.nblk == 1 || (a.N / 2) % 64 == 0, kErrShape, "%s: stacked output %lld (halves of 64s)", what,
                    (long long)a.N);
  }
  SMELB_CHECK_ARG(ws_bytes >= (int64_t)lin_layout(a.T, a.Kd, a.N).total, kErrWorkspace,
                  "%s: workspace %lld bytes, %lld needed", what, (long long)ws_bytes,
                  (long long)lin_layout(a.T, a.Kd, a.N).total);
  SMELB_CHECK_ARG(((uintptr_t)ws & 255) == 0, kErrArg, "%s: workspace must be 256-byte aligned", what);
  return kOk;
}

int lin_fwd(const LinArgs& a, void* y, void* xa, void* ws, int64_t ws_bytes, cudaStream_t st) {
  TRY(lin_check(a, ws, ws_bytes, "lora_linear_fwd"));
  SMELB_CHECK_ARG(y && (a.nblk == 0 || xa), kErrArg, "lora_linear_fwd: null output");
  if (a.T == 0) return kOk;
  const LinLayout lay = lin_layout(a.T, a.Kd, a.N);
  char* w8 = (char*)ws;
  int* tok = (int*)(w8 + lay.tok);
  TRY(set_counts(tok, 1, (int)a.T, a.T, st));
  const int r = (int)a.r, Kd = (int)a.Kd, N = (int)a.N, Nb = a.nblk ? N / a.nblk : N;
  if (a.nblk) {
    PackBatch pb;
    pb.n = 0;
    // xa_w [nblk r, Kd] = [A_0; A_1]; ext [N, 64]: rows of pair b hold s B_b in columns [b r, (b+1) r)
    TRY(pack(1, a.nblk * r, Kd, blk(a.A[0], 0, Kd, 1, 0, r, 0, Kd, 1.f),
             a.nblk > 1 ? blk(a.A[1], 0, Kd, 1, r, r, 0, Kd, 1.f) : no_blk(), w8 + lay.xa_w, pb));
    TRY(pack(1, N, kW64, blk(a.B[0], 0, r, 1, 0, Nb, 0, r, a.s),
             a.nblk > 1 ? blk(a.B[1], 0, r, 1, Nb, Nb, r, r, a.s) : no_blk(), w8 + lay.ext, pb));
    TRY(pack_batch(pb, st));
    Builder b;
    Problem& P = b.add();
    TRY(set_a_bf16(P, w8 + lay.xa_w, 1, a.nblk * r, Kd, false, false));
    TRY(set_b_tokens(P, a.x, a.T, Kd));
    groups(P, tok, nullptr, nullptr, nullptr, 1);
    out_bf16(P, xa, kW64);
    P.m_pad = kW64;  // the block's unused columns are written as zeros
    TRY(b.launch(st));
  }
  Builder b;
  Problem& P = b.add();
  TRY(set_a_bf16(P, a.w, 1, N, Kd, false, false));
  TRY(set_b_tokens(P, a.x, a.T, Kd));
  groups(P, tok, nullptr, nullptr, nullptr, 1);
  if (a.nblk) TRY(set_ext(P, w8 + lay.ext, 1, N, xa, a.T, false));
  out_bf16(P, y, N);
  return b.launch(st);
}

int lin_bwd(const LinArgs& a, const void* dy, const void* xa, void* dx, float* const gA[2], float* const gB[2], void* ws,
            int64_t ws_bytes, cudaStream_t st) {
  TRY(lin_check(a, ws, ws_bytes, "lora_linear_bwd"));
  SMELB_CHECK_ARG((a.T == 0 || dy) && (a.nblk == 0 || xa), kErrArg, "lora_linear_bwd: null input");
  if (a.T == 0) return kOk;
  const LinLayout lay = lin_layout(a.T, a.Kd, a.N);
  char* w8 = (char*)ws;
  int* tok = (int*)(w8 + lay.tok);
  TRY(set_counts(tok, 1, (int)a.T, a.T, st));
  const int r = (int)a.r, Kd = (int)a.Kd, N = (int)a.N, Nb = a.nblk ? N / a.nblk : N;
  void* dz = w8 + lay.dz;
  if (a.nblk) {
    PackBatch pb;
    pb.n = 0;
    // dz_w [nblk r, N]: pair b's rows hold s B_b^T over its output columns; dx_ext [Kd, 64] = [A_0^T | A_1^T | 0]
    TRY(pack(1, a.nblk * r, N, blk(a.B[0], 0, 1, r, 0, r, 0, Nb, a.s),
             a.nblk > 1 ? blk(a.B[1], 0, 1, r, r, r, Nb, Nb, a.s) : no_blk(), w8 + lay.dz_w, pb));
    TRY(pack(1, Kd, kW64, blk(a.A[0], 0, 1, Kd, 0, Kd, 0, r, 1.f),
             a.nblk > 1 ? blk(a.A[1], 0, 1, Kd, 0, Kd, r, r, 1.f) : no_blk(), w8 + lay.dx_ext, pb));
    TRY(pack_batch(pb, st));
    Builder b;
    Problem& P = b.add();
    TRY(set_a_bf16(P, w8 + lay.dz_w, 1, a.nblk * r, N, false, false));
    TRY(set_b_tokens(P, dy, a.T, N));
    groups(P, tok, nullptr, nullptr, nullptr, 1);
    out_bf16(P, dz, kW64);
    P.m_pad = kW64;
    TRY(b.launch(st));
  }
  Builder b;
  if (dx) {
    Problem& P = b.add();
    TRY(set_a_bf16(P, a.w, 1, N, Kd, true, false));
    TRY(set_b_tokens(P, dy, a.T, N));
    groups(P, tok, nullptr, nullptr, nullptr, 1);
    if (a.nblk) TRY(set_ext(P, w8 + lay.dx_ext, 1, Kd, dz, a.T, false));
    out_bf16(P, dx, Kd);
  }
  for (int k = 0; k < a.nblk; ++k) {
    if (gA[k]) {
      Problem& P = b.add();
      TRY(set_tokk(P, a.x, a.T, Kd, 0, Kd, dz, kW64, k * r, r, gA[k], 1, Kd, 0, 1.f));
      groups(P, tok, nullptr, nullptr, nullptr, 1);
    }
    if (gB[k]) {
      Problem& P = b.add();
      TRY(set_tokk(P, dy, a.T, N, k * Nb, Nb, xa, kW64, k * r, r, gB[k], r, 1, 0, a.s));
      groups(P, tok, nullptr, nullptr, nullptr, 1);
    }
  }
  return b.launch(st);
}

}  // namespace

// ================================================================================================== C ABI
extern "C" {

int smelb_version(void) { return kVersion; }

int smelb_last_error(char* buf, size_t len) {
  const char* e = smelb::last_error();
  const size_t n = strlen(e);
  if (buf && len) {
    const size_t c = n < len - 1 ? n : len - 1;
    memcpy(buf, e, c);
    buf[c] = 0;
  }
  return (int)n;
}

int smelb_set_device(int device) {
  static thread_local int current = -1;
  if (current != device) {
    SMELB_CUDA(cudaSetDevice(device));
    current = device;
  }
  return kOk;
}

int smelb_read_status(int device, int* status, int reset) {
  int detail[kStatusWords];
  const int rc = smelb_read_status_detail(device, detail, reset);
  if (rc == kOk && status) *status = detail[0];
  return rc;
}

int smelb_read_status_detail(int device, int* words, int reset) {
  SMELB_CHECK_ARG(words != nullptr, kErrArg, "read_status: null output");
  int prev = 0;
  SMELB_CUDA(cudaGetDevice(&prev));
  SMELB_CUDA(cudaSetDevice(device));
  int* w = device_status(device);
  SMELB_CHECK_ARG(w != nullptr, kErrCuda, "read_status: no status word");
  SMELB_CUDA(cudaDeviceSynchronize());
  SMELB_CUDA(cudaMemcpy(words, w, kStatusWords * sizeof(int), cudaMemcpyDeviceToHost));
  if (reset) SMELB_CUDA(cudaMemset(w, 0, kStatusWords * sizeof(int)));
  SMELB_CUDA(cudaSetDevice(prev));
  return kOk;
}

int smelb_int4_dequant(const void* q, const void* scale, const void* zero, void* out, int64_t rows, int64_t k,
                       int64_t groups, int out_fp32, void* stream) {
  SMELB_CHECK_ARG(q && scale && zero && out, kErrArg, "int4_dequant: null pointer");
  return int4_dequant(q, scale, zero, out, rows, (int)k, (int)groups, out_fp32 != 0, (cudaStream_t)stream);
}

int smelb_int4_quantize(const void* w, int w_fp32, int64_t rows, int64_t k, const float* clip, int n_clip, void* q,
                        void* scale, void* zero, void* stream) {
  SMELB_CHECK_ARG(w && clip && q && scale && zero, kErrArg, "int4_quantize: null pointer");
  return int4_quantize(w, w_fp32 != 0, rows, (int)k, clip, n_clip, q, scale, zero, (cudaStream_t)stream);
}

int smelb_int4_pack_sz(const void* scale, const void* zero, uint32_t* sz_t, int64_t nw, int64_t rows,
                       int64_t groups, void* stream) {
  SMELB_CHECK_ARG(scale && zero && sz_t, kErrArg, "int4_pack_sz: null pointer");
  return int4_pack_sz(scale, zero, sz_t, nw, (int)rows, (int)groups, (cudaStream_t)stream);
}

int smelb_router_topk(const void* logits, int64_t ld, int64_t T, int64_t E, int64_t K, float* probs, void* topv,
                      int topv_fp32, int64_t* topi, const void* per_expert_scale, void* stream) {
  SMELB_CHECK_ARG(logits && probs && topv && topi, kErrArg, "router_topk: null pointer");
  return router_topk(logits, ld, (int)T, (int)E, (int)K, probs, topv, topv_fp32 != 0, (long long*)topi,
                     per_expert_scale, (cudaStream_t)stream);
}

int smelb_router_bwd(const void* dtopv, int dtopv_fp32, const float* probs, const int64_t* topi,
                     const void* per_expert_scale, int64_t T, int64_t E, int64_t K, void* dlogits, int64_t ld,
                     void* stream) {
  SMELB_CHECK_ARG(probs && topi && dlogits, kErrArg, "router_bwd: null pointer");
  return router_bwd(dtopv, dtopv_fp32 != 0, nullptr, probs, (const long long*)topi, per_expert_scale, (int)T,
                    (int)E, (int)K, dlogits, ld, (cudaStream_t)stream);
}

int smelb_dispatch_plan(const int64_t* topi, int64_t T, int64_t K, int64_t E, const uint8_t* sel_mask, int64_t pad,
                        int32_t* counts, int32_t* gcounts, int32_t* offsets, int32_t* row_of, int32_t* src_of,
                        int64_t* order, int32_t* total, void* stream) {
  SMELB_CHECK_ARG(topi && counts && gcounts && offsets && row_of && src_of && order && total, kErrArg,
                  "dispatch_plan: null pointer");
  return dispatch_plan((const long long*)topi, T * K, (int)E, sel_mask, (int)pad, counts, gcounts, offsets, row_of,
                       src_of, (long long*)order, total, (cudaStream_t)stream);
}

int smelb_dispatch_plan_ws(const int64_t* topi, int64_t T, int64_t K, int64_t E, const uint8_t* sel_mask,
                           int64_t pad, int32_t* counts, int32_t* gcounts, int32_t* offsets, int32_t* row_of,
                           int32_t* src_of, int64_t* order, int32_t* total, int32_t* workspace,
                           int64_t workspace_ints, void* stream) {
  SMELB_CHECK_ARG(topi && counts && gcounts && offsets && row_of && src_of && order && total && workspace, kErrArg,
                  "dispatch_plan_ws: null pointer");
  return dispatch_plan_mt((const long long*)topi, T * K, (int)E, sel_mask, (int)pad, counts, gcounts, offsets, row_of,
                          src_of, (long long*)order, total, workspace, workspace_ints, (cudaStream_t)stream);
}

int smelb_gather_rows(const void* x, int64_t H, int64_t K, const int32_t* src_of, const int32_t* total,
                      int64_t max_rows, void* xs, void* stream) {
  SMELB_CHECK_ARG(x && src_of && total && xs, kErrArg, "gather_rows: null pointer");
  return gather_rows(x, (int)H, (int)K, src_of, total, max_rows, xs, (cudaStream_t)stream);
}

int smelb_combine_fwd(const void* y, const int32_t* row_of, const void* topv, int topv_fp32, int64_t T, int64_t K,
                      int64_t H, void* out, void* stream) {
  SMELB_CHECK_ARG(y && row_of && topv && out, kErrArg, "combine_fwd: null pointer");
  return combine_fwd(y, row_of, topv, topv_fp32 != 0, (int)T, (int)K, (int)H, nullptr, nullptr, out,
                     (cudaStream_t)stream);
}

int smelb_combine_bwd(const void* g, const void* y, const int32_t* src_of, const int32_t* total, int64_t max_rows,
                      const void* topv, int topv_fp32, int64_t K, int64_t H, void* dy, void* dtopv, void* stream) {
  SMELB_CHECK_ARG(g && y && src_of && total && topv && dy, kErrArg, "combine_bwd: null pointer");
  SMELB_CHECK_ARG(K >= 1 && K <= 32 && H % 8 == 0, kErrShape, "combine_bwd: K=%lld H=%lld", (long long)K, (long long)H);
  return combine_bwd_rows(g, y, src_of, total, max_rows, topv, topv_fp32 != 0, (int)K, (int)H, dy, dtopv,
                          (cudaStream_t)stream);
}

int smelb_gather_rows_bwd(const void* dxs, const int32_t* row_of, int64_t T, int64_t K, int64_t H, void* dx,
                          void* stream) {
  SMELB_CHECK_ARG(dxs && row_of && dx, kErrArg, "gather_rows_bwd: null pointer");
  SMELB_CHECK_ARG(K >= 1 && K <= 32, kErrShape, "gather_rows_bwd: K=%lld", (long long)K);
  return dx_reduce(dxs, row_of, (int)K, (int)T, (int)H, nullptr, nullptr, nullptr, nullptr, dx, (cudaStream_t)stream);
}

int smelb_rmsnorm_fwd(const void* x, const void* h_add, const void* w, int w_mode, const void* post_scale,
                      float post_mul, float eps, int64_t rows, int64_t C, void* s_out, void* y, float* rstd_out,
                      void* stream) {
  SMELB_CHECK_ARG(x && y, kErrArg, "rmsnorm_fwd: null pointer");
  SMELB_CHECK_ARG(w_mode >= 0 && w_mode <= 2, kErrArg, "rmsnorm_fwd: w_mode %d", w_mode);
  NormArgs a{(const bf16*)x, (const bf16*)h_add, (const bf16*)w, (const bf16*)post_scale, post_mul, w_mode, eps,
             (long long)rows, (int)C, (bf16*)s_out, (bf16*)y, rstd_out};
  return rmsnorm_fwd(a, (cudaStream_t)stream);
}

int smelb_rmsnorm_bwd(const void* dy, const void* x, const void* w, int w_mode, const void* post_scale,
                      float post_mul, const float* rstd, const void* ds, int64_t rows, int64_t C, void* dx,
                      void* stream) {
  SMELB_CHECK_ARG(dy && x && rstd && dx, kErrArg, "rmsnorm_bwd: null pointer");
  SMELB_CHECK_ARG(w_mode >= 0 && w_mode <= 2, kErrArg, "rmsnorm_bwd: w_mode %d", w_mode);
  NormBwdArgs a{(const bf16*)dy, (const bf16*)x, (const bf16*)w, (const bf16*)post_scale, post_mul, w_mode, rstd,
                (const bf16*)ds, (long long)rows, (int)C, (bf16*)dx};
  return rmsnorm_bwd(a, (cudaStream_t)stream);
}

int smelb_frozen_experts_fwd(const void* xs, int64_t rows, int64_t H, int64_t I, const int32_t* counts, int64_t E,
                             const void* gu_q, const uint32_t* gu_sz, const void* dn_q, const uint32_t* dn_sz,
                             int act, void* h_save, void* a_buf, void* out, void* stream) {
  SMELB_CHECK_ARG(gu_q && gu_sz && dn_q && dn_sz, kErrArg, "frozen_experts_fwd: null pointer");
  const FrozenBank bank{Int4Mat{gu_q, gu_sz, (int)E, (int)(2 * I), (int)H}, Int4Mat{dn_q, dn_sz, (int)E, (int)H, (int)I},
                        nullptr, nullptr, (int)E};
  return frozen_fwd(bank, xs, rows, H, I, counts, E, act, h_save, a_buf, out, (cudaStream_t)stream, nullptr);
}

int smelb_frozen_experts_bf16_fwd(const void* xs, int64_t rows, int64_t H, int64_t I, const int32_t* counts,
                                  int64_t E, const void* gate_up, const void* down, int act, void* h_save, void* a_buf,
                                  void* out, void* stream) {
  SMELB_CHECK_ARG(gate_up && down, kErrArg, "frozen_experts_bf16_fwd: null pointer");
  const FrozenBank bank{Int4Mat{}, Int4Mat{}, gate_up, down, (int)E};
  return frozen_fwd(bank, xs, rows, H, I, counts, E, act, h_save, a_buf, out, (cudaStream_t)stream, nullptr);
}

int smelb_frozen_experts_bwd(const void* xs, const void* dy, int64_t rows, int64_t H, int64_t I,
                             const int32_t* counts, int64_t E, const void* gu_q, const uint32_t* gu_sz,
                             const void* dn_q, const uint32_t* dn_sz, int act, const void* h, void* h_buf,
                             void* dh_buf, void* dx, void* stream) {
  SMELB_CHECK_ARG(gu_q && gu_sz && dn_q && dn_sz, kErrArg, "frozen_experts_bwd: null pointer");
  const FrozenBank bank{Int4Mat{gu_q, gu_sz, (int)E, (int)(2 * I), (int)H}, Int4Mat{dn_q, dn_sz, (int)E, (int)H, (int)I},
                        nullptr, nullptr, (int)E};
  return frozen_bwd(bank, xs, dy, rows, H, I, counts, E, act, h, h_buf, dh_buf, dx, (cudaStream_t)stream);
}

int smelb_frozen_experts_bf16_bwd(const void* xs, const void* dy, int64_t rows, int64_t H, int64_t I,
                                  const int32_t* counts, int64_t E, const void* gate_up, const void* down, int act,
                                  const void* h, void* h_buf, void* dh_buf, void* dx, void* stream) {
  SMELB_CHECK_ARG(gate_up && down, kErrArg, "frozen_experts_bf16_bwd: null pointer");
  const FrozenBank bank{Int4Mat{}, Int4Mat{}, gate_up, down, (int)E};
  return frozen_bwd(bank, xs, dy, rows, H, I, counts, E, act, h, h_buf, dh_buf, dx, (cudaStream_t)stream);
}

int smelb_int4_dequant_stepwise(const void* q, const void* scale, const void* zero, void* out, int64_t rows,
                                int64_t k, int64_t groups, int out_fp32, void* stream) {
  SMELB_CHECK_ARG(q && scale && zero && out, kErrArg, "int4_dequant_stepwise: null pointer");
  return int4_dequant(q, scale, zero, out, rows, (int)k, (int)groups, out_fp32 != 0, (cudaStream_t)stream, true);
}

int smelb_lora_merge(const void* w, int w_fp32, int64_t rows, int64_t cols, const float* B, const float* A, int64_t r,
                     float scale, void* out, void* stream) {
  SMELB_CHECK_ARG(w && B && A && out, kErrArg, "lora_merge: null pointer");
  SMELB_CHECK_ARG(rows >= 0 && cols >= 0 && r >= 1 && rows < (1LL << 31) && cols < (1LL << 31) && r <= 4096, kErrShape,
                  "lora_merge: rows=%lld cols=%lld r=%lld", (long long)rows, (long long)cols, (long long)r);
  return lora_merge(w, w_fp32 != 0, B, A, (int)rows, (int)cols, (int)r, scale, out, (cudaStream_t)stream);
}

int64_t smelb_lora_linear_workspace_bytes(int64_t T, int64_t in_features, int64_t out_features) {
  if (T < 0 || in_features <= 0 || out_features <= 0) return 0;
  return (int64_t)lin_layout(T, in_features, out_features).total;
}

int smelb_lora_linear_fwd(const void* x, int64_t T, int64_t in_features, const void* w, int64_t out_features,
                          const float* A0, const float* B0, const float* A1, const float* B1, int64_t r, float scale,
                          void* y, void* xa, void* workspace, int64_t workspace_bytes, void* stream) {
  SMELB_CHECK_ARG((A0 == nullptr) == (B0 == nullptr) && (A1 == nullptr) == (B1 == nullptr) && (A0 || !A1), kErrArg,
                  "lora_linear_fwd: give A and B together, the second pair only with the first");
  const LinArgs a{x, T, in_features, out_features, r, w, {A0, A1}, {B0, B1}, A0 ? (A1 ? 2 : 1) : 0, scale};
  return lin_fwd(a, y, xa, workspace, workspace_bytes, (cudaStream_t)stream);
}

int smelb_lora_linear_bwd(const void* x, const void* dy, int64_t T, int64_t in_features, const void* w,
                          int64_t out_features, const float* A0, const float* B0, const float* A1, const float* B1,
                          int64_t r, float scale, const void* xa, void* dx, float* gA0, float* gB0, float* gA1,
                          float* gB1, void* workspace, int64_t workspace_bytes, void* stream) {
  SMELB_CHECK_ARG((A0 == nullptr) == (B0 == nullptr) && (A1 == nullptr) == (B1 == nullptr) && (A0 || !A1), kErrArg,
                  "lora_linear_bwd: give A and B together, the second pair only with the first");
  SMELB_CHECK_ARG(x || T == 0, kErrArg, "lora_linear_bwd: null x");
  const LinArgs a{x, T, in_features, out_features, r, w, {A0, A1}, {B0, B1}, A0 ? (A1 ? 2 : 1) : 0, scale};
  float* const gA[2] = {gA0, gA1};
  float* const gB[2] = {gB0, gB1};
  return lin_bwd(a, dy, xa, dx, gA, gB, workspace, workspace_bytes, (cudaStream_t)stream);
}

size_t smelb_moe_layer_size(void) { return sizeof(smelb_moe_layer); }

long long smelb_launch_count(void) { return smelb::launch_count(); }

int64_t smelb_set_gemv_rows(int64_t rows) {
  return g_gemv_rows.exchange(rows < 0 ? 0 : (long long)rows);
}

int smelb_gemm_timing(int enable) {
  smelb::set_gemm_timing(enable != 0);
  return kOk;
}

int smelb_gemm_timing_read(double* ms_total, long long* launches) {
  SMELB_CHECK_ARG(ms_total && launches, kErrArg, "gemm_timing_read: null output");
  return smelb::read_gemm_timing(ms_total, launches);
}

int smelb_moe_layer_fwd(const smelb_moe_layer* L) {
  SMELB_CHECK_ARG(L != nullptr, kErrArg, "moe_layer_fwd: null layer");
  return layer_fwd(*L);
}

int smelb_moe_layer_bwd(const smelb_moe_layer* L) {
  SMELB_CHECK_ARG(L != nullptr, kErrArg, "moe_layer_bwd: null layer");
  return layer_bwd(*L);
}

}  // extern "C"

// ------------------------------------------------------------------------------------- no-allocation variant
// smelb_frozen_experts_fwd with its intermediate (the activated gate*up rows, bf16 [rows, I]) and its wait-timeout
// status words in one file-scope device array instead of caller scratch and the lazily allocated per-device status
// word. Layout of the array: bytes [0, 256) status words (4 ints used, cleared by every call), bytes
// [256, 256 + SMELB_NOALLOC_SCRATCH_BYTES) the intermediate. All calls on a device share the array.
static constexpr size_t kNoAllocHead = 256;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocHead + SMELB_NOALLOC_SCRATCH_BYTES];
namespace {
std::mutex g_noalloc_mu;
unsigned char* g_noalloc_ptr[64] = {nullptr};

// Device address of g_noalloc_scratch on `dev` (the current device), resolved once per device.
int noalloc_scratch(int dev, unsigned char** out) {
  SMELB_CHECK_ARG(dev >= 0 && dev < 64, kErrArg, "frozen_experts_fwd_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    SMELB_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_noalloc_ptr[dev] = (unsigned char*)p;
  }
  *out = g_noalloc_ptr[dev];
  return kOk;
}
}  // namespace

extern "C" int smelb_frozen_experts_fwd_noalloc(const void* xs, int64_t rows, int64_t H, int64_t I,
                                                const int32_t* counts, int64_t E, const void* gu_q,
                                                const uint32_t* gu_sz, const void* dn_q, const uint32_t* dn_sz,
                                                int act, void* h_save, void* out, void* stream) {
  SMELB_CHECK_ARG(xs && counts && gu_q && gu_sz && dn_q && dn_sz && out, kErrArg,
                  "frozen_experts_fwd_noalloc: null pointer");
  SMELB_CHECK_ARG(H % 64 == 0 && I % 64 == 0 && E >= 1 && E <= kMaxGroups && rows >= 0, kErrShape,
                  "frozen_experts_fwd_noalloc: rows=%lld H=%lld I=%lld E=%lld", (long long)rows, (long long)H,
                  (long long)I, (long long)E);
  SMELB_CHECK_ARG(act == SMELB_ACT_SILU || act == SMELB_ACT_GELU_TANH, kErrArg, "unknown activation %d", act);
  SMELB_CHECK_ARG(rows <= (int64_t)(SMELB_NOALLOC_SCRATCH_BYTES / 2) / (I > 0 ? I : 1), kErrShape,
                  "frozen_experts_fwd_noalloc: rows*I*2 = %lld bytes exceeds the %lld-byte scratch (max rows %lld "
                  "at I=%lld)",
                  (long long)rows * (long long)I * 2, (long long)SMELB_NOALLOC_SCRATCH_BYTES,
                  (long long)(SMELB_NOALLOC_SCRATCH_BYTES / 2 / I), (long long)I);
  if (rows == 0) return kOk;
  int dev = 0;
  SMELB_CUDA(cudaGetDevice(&dev));
  unsigned char* scratch = nullptr;
  TRY(noalloc_scratch(dev, &scratch));
  cudaStream_t st = (cudaStream_t)stream;
  int* err = (int*)scratch;
  SMELB_CUDA(cudaMemsetAsync(err, 0, kNoAllocHead, st));
  const FrozenBank bank{Int4Mat{gu_q, gu_sz, (int)E, (int)(2 * I), (int)H}, Int4Mat{dn_q, dn_sz, (int)E, (int)H, (int)I},
                        nullptr, nullptr, (int)E};
  return frozen_fwd(bank, xs, rows, H, I, counts, E, act, h_save, scratch + kNoAllocHead, out, st, err);
}

// Status words of the last smelb_frozen_experts_fwd_noalloc call on `device`: synchronizes the device and copies the
// head of the shared array (no allocation). words[0] is 0, or the code of a bounded device-side wait that gave up
// inside that call (its output is then incomplete); words[1..3] block, tile and k-block.
extern "C" int smelb_frozen_experts_fwd_noalloc_status(int device, int* words, int reset) {
  SMELB_CHECK_ARG(words != nullptr, kErrArg, "frozen_experts_fwd_noalloc_status: null output");
  int prev = 0;
  SMELB_CUDA(cudaGetDevice(&prev));
  SMELB_CUDA(cudaSetDevice(device));
  unsigned char* scratch = nullptr;
  int rc = noalloc_scratch(device, &scratch);
  if (rc == kOk) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(words, scratch, kStatusWords * sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && reset) e = cudaMemset(scratch, 0, kStatusWords * sizeof(int));
    if (e != cudaSuccess) {
      set_last_error("frozen_experts_fwd_noalloc_status: %s", cudaGetErrorString(e));
      rc = kErrCuda;
    }
  }
  SMELB_CUDA(cudaSetDevice(prev));
  return rc;
}

// ---------------------------------------------------------------------------------------------------- chunked CE
// smel/loss.py:130-146 _ChunkedCE.forward with smel/loss.py:50-92 _ce_chunk: one pass over the vocabulary, the
// online state (running max / sum, target logit and row, fp32 gradient accumulator) kept for every row. The loops
// run vocabulary-outer, token-chunk-inner, so an int8 head is dequantised once per call and each vocabulary chunk's
// rows are read while they are hot; every row still sees the vocabulary chunks in the reference's order, so the
// per-row results are the reference's token chunk by token chunk. Per (vocabulary chunk, token chunk):
//   GEMM 1  lg[n, Vcp] = bf16(h @ Wc^T)                         (A = Wc K-major, tokens as B, the MoE GEMM engine)
//   rows    online max / sum, target capture, p = exp(z - m) * cap'(z) in bf16 over lg in place
//   GEMM 2  part[s][n, H] = p[:, ks] @ Wc[ks]                  (A = Wc MN-major, the chunk split along k into
//                                                               nsplit fp32 partials so the tiles fill the SMs)
//   acc     acc = acc * r + sum_s part[s]
// then loss_rows and gh for every row, and the loss.
namespace {

constexpr int kCeMaxSplit = 4;

size_t ce_align(size_t x) { return (x + 255) & ~size_t(255); }

struct CeLayout {
  size_t tok, lg, parts, acc, tgt_row, m, s, r, tlog, tdrv, wc, total;
};

// N rows of state, token chunks of tc rows, vocabulary chunks of vc rows
CeLayout ce_layout(long long N, long long tc, long long H, long long vc, bool int8, bool grad) {
  const long long vcp = (vc + 63) / 64 * 64;
  CeLayout L{};
  size_t o = 0;
  L.tok = o;      o += ce_align((size_t)4 * ((N + tc - 1) / tc));  // one token count per token chunk
  L.lg = o;       o += ce_align((size_t)tc * vcp * 2);
  L.parts = o;    o += grad ? ce_align((size_t)kCeMaxSplit * tc * H * 4) : 0;
  L.acc = o;      o += grad ? ce_align((size_t)N * H * 4) : 0;
  L.tgt_row = o;  o += grad ? ce_align((size_t)N * H * 4) : 0;
  L.m = o;        o += ce_align((size_t)N * 4);
  L.s = o;        o += ce_align((size_t)N * 4);
  L.r = o;        o += ce_align((size_t)N * 4);
  L.tlog = o;     o += ce_align((size_t)N * 4);
  L.tdrv = o;     o += ce_align((size_t)N * 4);
  L.wc = o;       o += int8 ? ce_align((size_t)vc * H * 2) : 0;
  L.total = o;
  return L;
}

// Number of k-splits of GEMM 2 whose tiles best fill whole waves of the SMs (fewest splits on a tie).
int ce_splits(long long n, long long H, int vcp, int sms) {
  const long long tiles = ((H + 127) / 128) * ((n + kMaxBN - 1) / kMaxBN);
  int best = 1;
  double best_fill = 0.0;
  for (int s = 1; s <= kCeMaxSplit && 64 * s <= vcp; ++s) {
    const long long t = tiles * s;
    const double fill = (double)t / (double)(((t + sms - 1) / sms) * sms);
    if (fill > best_fill + 1e-9) {
      best_fill = fill;
      best = s;
    }
  }
  return best;
}

CeState ce_state_at(const CeState& S, long long t0, long long H) {
  return CeState{S.m + t0,    S.s + t0,    S.r + t0, S.tlog + t0, S.tdrv + t0,
                 S.acc ? S.acc + t0 * H : nullptr, S.tgt_row ? S.tgt_row + t0 * H : nullptr};
}

}  // namespace

int smelb_int8_rows_quantize(const void* w, int w_fp32, int64_t rows, int64_t H, void* q, void* scale,
                              void* stream) {
  SMELB_CHECK_ARG(w && q && scale, kErrArg, "int8_rows_quantize: null pointer");
  SMELB_CHECK_ARG(H > 0 && H <= (1 << 30), kErrShape, "int8_rows_quantize: H=%lld", (long long)H);
  return int8_rows_quantize(w, w_fp32 != 0, rows, (int)H, q, scale, (cudaStream_t)stream);
}

int smelb_int8_rows_dequant(const void* q, const void* scale, int64_t rows, int64_t H, void* out, int out_fp32,
                            void* stream) {
  SMELB_CHECK_ARG(q && scale && out, kErrArg, "int8_rows_dequant: null pointer");
  SMELB_CHECK_ARG(H > 0 && H <= (1 << 30), kErrShape, "int8_rows_dequant: H=%lld", (long long)H);
  return int8_rows_dequant(q, scale, rows, (int)H, out, (cudaStream_t)stream, out_fp32 != 0);
}

int64_t smelb_chunked_ce_workspace_bytes(int64_t N, int64_t token_chunk, int64_t H, int64_t vocab_chunk, int int8,
                                         int need_grad) {
  if (N <= 0 || token_chunk <= 0 || H <= 0 || vocab_chunk <= 0) return 256;
  return (int64_t)ce_layout(N, std::min<int64_t>(token_chunk, N), H, vocab_chunk, int8 != 0, need_grad != 0).total;
}

int smelb_chunked_ce(const void* h, const int64_t* tgt, int64_t N, int64_t H, const void* w, const void* q,
                     const void* q_scale, int64_t V, int64_t vocab_chunk, int64_t token_chunk, float softcap,
                     float denom, float* loss_rows, float* loss, void* gh, void* workspace, int64_t workspace_bytes,
                     void* stream) {
  SMELB_CHECK_ARG(tgt && loss_rows && loss && workspace && (N == 0 || h), kErrArg, "chunked_ce: null pointer");
  SMELB_CHECK_ARG((w != nullptr) != (q != nullptr) && (q == nullptr || q_scale != nullptr), kErrArg,
                  "chunked_ce: pass exactly one of the bf16 head (w) or the int8 head (q, q_scale)");
  SMELB_CHECK_ARG(H > 0 && H % 64 == 0 && H <= 65536, kErrShape, "chunked_ce: H=%lld (a multiple of 64 is required)",
                  (long long)H);
  SMELB_CHECK_ARG(N >= 0 && N <= (1LL << 31) - 1 && V > 0 && vocab_chunk > 0 && vocab_chunk <= (1 << 24) &&
                      token_chunk > 0 && V < (1LL << 40),
                  kErrShape, "chunked_ce: N=%lld V=%lld vocab_chunk=%lld token_chunk=%lld", (long long)N,
                  (long long)V, (long long)vocab_chunk, (long long)token_chunk);
  SMELB_CHECK_ARG(softcap >= 0.f, kErrArg, "chunked_ce: softcap=%g", (double)softcap);
  cudaStream_t st = (cudaStream_t)stream;
  if (N == 0) return ce_loss_sum(loss_rows, 0, denom, loss, st);
  const bool int8 = q != nullptr;
  const bool need_grad = gh != nullptr;
  const long long tc = std::min<long long>(token_chunk, N);
  const long long vc_max = std::min<long long>(vocab_chunk, V);
  const CeLayout lay = ce_layout(N, tc, H, vc_max, int8, need_grad);
  SMELB_CHECK_ARG(workspace_bytes >= (int64_t)lay.total, kErrWorkspace,
                  "chunked_ce: workspace %lld bytes, %lld needed", (long long)workspace_bytes, (long long)lay.total);
  SMELB_CHECK_ARG(((uintptr_t)workspace & 255) == 0 && ((uintptr_t)h & 15) == 0 && (int8 || ((uintptr_t)w & 15) == 0),
                  kErrArg, "chunked_ce: workspace must be 256-byte aligned, h and w 16-byte aligned");
  char* ws = (char*)workspace;
  int* tok = (int*)(ws + lay.tok);
  bf16* lg = (bf16*)(ws + lay.lg);
  float* parts = need_grad ? (float*)(ws + lay.parts) : nullptr;
  const CeState S{(float*)(ws + lay.m),    (float*)(ws + lay.s),   (float*)(ws + lay.r), (float*)(ws + lay.tlog),
                  (float*)(ws + lay.tdrv), need_grad ? (float*)(ws + lay.acc) : nullptr,
                  need_grad ? (float*)(ws + lay.tgt_row) : nullptr};
  int dev = 0;
  SMELB_CUDA(cudaGetDevice(&dev));
  const int sms = num_sms(dev);
  TRY(ce_init(S, N, (int)H, st));
  TRY(set_counts(tok, (int)((N + tc - 1) / tc), (int)tc, N, st));
  for (long long v0 = 0; v0 < V; v0 += vocab_chunk) {
    const int Vc = (int)std::min<long long>(vocab_chunk, V - v0);
    const int vcp = (Vc + 63) / 64 * 64;
    const void* wc;
    if (int8) {
      TRY(int8_rows_dequant((const int8_t*)q + v0 * H, (const bf16*)q_scale + v0, Vc, (int)H, ws + lay.wc, st));
      wc = ws + lay.wc;
    } else {
      wc = (const bf16*)w + v0 * H;
    }
    for (long long t0 = 0; t0 < N; t0 += tc) {
      const long long n = std::min<long long>(tc, N - t0);
      const bf16* hc = (const bf16*)h + t0 * H;
      const CeState Sc = ce_state_at(S, t0, H);
      const int* cnt = tok + t0 / tc;
      {
        Builder b;
        Problem& P = b.add();
        TRY(set_a_bf16(P, wc, 1, Vc, (int)H, false, false));
        TRY(set_b_tokens(P, hc, n, (int)H));
        groups(P, cnt, nullptr, nullptr, nullptr, 1);
        out_bf16(P, lg, vcp);
        P.n_inner = 1;  // the head tile is shared by the chunk's token tiles through L2
        TRY(b.launch(st));
      }
      TRY(ce_rows(lg, vcp, Vc, v0, (const long long*)tgt + t0, softcap, need_grad, wc, (int)H, Sc, n, st));
      if (!need_grad) continue;
      const int ns = ce_splits(n, H, vcp, sms);
      const int kstep = ((vcp / 64 + ns - 1) / ns) * 64;
      int np = 0;
      {
        Builder b;
        for (int k0 = 0; k0 < vcp; k0 += kstep, ++np) {
          const int kk = std::min(kstep, vcp - k0);
          const int rows = std::min(Vc, k0 + kk) - k0;  // >= 1: only the last 63 columns of vcp can lie past Vc
          Problem& P = b.add();
          TRY(set_a_bf16(P, (const bf16*)wc + (long long)k0 * H, 1, rows, (int)H, true, false));
          P.K = kk;
          P.mode = kTokN;
          P.BN = kMaxBN;
          TRY(make_tmap_2d(&P.tmB32, lg + k0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, n, kk, (uint64_t)vcp * 2, 64, 32,
                           128));
          TRY(make_tmap_2d(&P.tmB, lg + k0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, n, kk, (uint64_t)vcp * 2, 64, 64,
                           128));
          groups(P, cnt, nullptr, nullptr, nullptr, 1);
          P.epi = kEpiStoreF32;
          P.C = parts + (long long)np * n * H;
          P.c_sn = H;
          P.c_sm = 1;
        }
        TRY(b.launch(st));
      }
      TRY(ce_acc(parts, np, Sc, n, (int)H, st));
    }
  }
  TRY(ce_finish(S, N, (int)H, denom, loss_rows, need_grad ? gh : nullptr, st));
  return ce_loss_sum(loss_rows, N, denom, loss, st);
}

namespace {
// workspace of smelb_lm_logits: the token count, the chunk's bf16 logits [N, Vcp] and (int8 head) its bf16 rows
struct LogitsLayout {
  size_t tok, lg, wc, total;
};
LogitsLayout logits_layout(long long N, long long H, long long vocab_chunk, bool int8) {
  const long long vcp = (vocab_chunk + 63) / 64 * 64;
  LogitsLayout L{};
  L.tok = 0;
  L.lg = ce_align(4);
  L.wc = L.lg + ce_align((size_t)N * vcp * 2);
  L.total = L.wc + (int8 ? ce_align((size_t)vocab_chunk * H * 2) : 0);
  return L;
}
}  // namespace

int64_t smelb_lm_logits_workspace_bytes(int64_t N, int64_t H, int64_t vocab_chunk, int int8) {
  if (N <= 0 || H <= 0 || vocab_chunk <= 0) return 0;
  return (int64_t)logits_layout(N, H, vocab_chunk, int8 != 0).total;
}

int smelb_lm_logits(const void* h, int64_t N, int64_t H, const void* w, const void* q, const void* q_scale, int64_t V,
                    int64_t vocab_chunk, float softcap, float* out, void* workspace, int64_t workspace_bytes,
                    void* stream) {
  SMELB_CHECK_ARG(out && workspace && (N == 0 || h), kErrArg, "lm_logits: null pointer");
  SMELB_CHECK_ARG((w != nullptr) != (q != nullptr) && (q == nullptr || q_scale != nullptr), kErrArg,
                  "lm_logits: pass exactly one of the bf16 head (w) or the int8 head (q, q_scale)");
  SMELB_CHECK_ARG(H > 0 && H % 64 == 0 && H <= 65536 && N >= 0 && N <= (1LL << 31) - 1 && V > 0 && vocab_chunk > 0 &&
                      vocab_chunk <= (1 << 24),
                  kErrShape, "lm_logits: N=%lld H=%lld V=%lld vocab_chunk=%lld", (long long)N, (long long)H,
                  (long long)V, (long long)vocab_chunk);
  SMELB_CHECK_ARG(softcap >= 0.f, kErrArg, "lm_logits: softcap=%g", (double)softcap);
  if (N == 0) return kOk;
  cudaStream_t st = (cudaStream_t)stream;
  const bool int8 = q != nullptr;
  const LogitsLayout lay = logits_layout(N, H, std::min<long long>(vocab_chunk, V), int8);
  SMELB_CHECK_ARG(workspace_bytes >= (int64_t)lay.total, kErrWorkspace, "lm_logits: workspace %lld bytes, %lld needed",
                  (long long)workspace_bytes, (long long)lay.total);
  SMELB_CHECK_ARG(((uintptr_t)workspace & 255) == 0 && ((uintptr_t)h & 15) == 0 && (int8 || ((uintptr_t)w & 15) == 0),
                  kErrArg, "lm_logits: workspace must be 256-byte aligned, h and w 16-byte aligned");
  char* ws = (char*)workspace;
  int* tok = (int*)(ws + lay.tok);
  bf16* lg = (bf16*)(ws + lay.lg);
  TRY(set_counts(tok, 1, (int)N, N, st));
  for (long long v0 = 0; v0 < V; v0 += vocab_chunk) {
    const int Vc = (int)std::min<long long>(vocab_chunk, V - v0);
    const int vcp = (Vc + 63) / 64 * 64;
    const void* wc;
    if (int8) {
      TRY(int8_rows_dequant((const int8_t*)q + v0 * H, (const bf16*)q_scale + v0, Vc, (int)H, ws + lay.wc, st));
      wc = ws + lay.wc;
    } else {
      wc = (const bf16*)w + v0 * H;
    }
    Builder b;
    Problem& P = b.add();
    TRY(set_a_bf16(P, wc, 1, Vc, (int)H, false, false));
    TRY(set_b_tokens(P, h, N, (int)H));
    groups(P, tok, nullptr, nullptr, nullptr, 1);
    out_bf16(P, lg, vcp);
    P.n_inner = 1;
    TRY(b.launch(st));
    TRY(ce_logits_out(lg, vcp, Vc, N, softcap, out + v0, V, st));
  }
  return kOk;
}
