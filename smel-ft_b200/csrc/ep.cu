// Expert-parallel exchange of the MoE layer over peer memory (NVLink), with the C ABI of include/smelb.h.
//
// Every rank of an expert-parallel group owns one region of device memory (cudaMalloc'd by the library, mapped into
// every peer by CUDA IPC). A rank is the source of its own tokens and the owner of its share of the experts. Per
// layer call there are four exchanges, each through its own buffer b of the region:
//   b = 0  forward dispatch: the source's token rows, de-duplicated per destination (a token goes once to each rank
//          that owns at least one of its experts), with the (local expert, k, weight) entries of every row
//   b = 1  forward return: per received row, the owner's partial combine sum_j weight_j * y_j over its entries
//   b = 2  backward dispatch: the upstream gradient rows of the same token rows
//   b = 3  backward return: per received row the summed dX of its entries, and d weight per entry
// A sender writes into its own region and publishes; the readers pull from the sender's region and acknowledge. The
// synchronisation is device-side (epoch counters per buffer, release / acquire at system scope), so a whole layer
// step can be captured in a CUDA graph and no call synchronises with the host. Every wait is bounded: after
// SMELB_WAIT_NS it records kDevErrEpWait in the status word and returns.
#include <cstring>

#include "../../include/smelb.h"
#include "common.cuh"
#include "host.h"
#include "kernels.h"

namespace smelb {

constexpr int kEpMaxRanks = 8;
constexpr int kEpMaxK = 16;
constexpr int kDevErrEpWait = 13;     // a peer's flag did not arrive in time
constexpr int kDevErrEpCapacity = 14; // more dispatch entries than the owner's capacity

// ------------------------------------------------------------------------------------------ region layout
struct EpLayout {
  size_t ready, done, send_epoch, recv_epoch, counts, nent, tcnt, meta, wts, eoff, dwts, rows[4], total;
};

constexpr int kPlanTile = 256;  // tokens per block of the source-side plan

static size_t ep_al(size_t x) { return (x + 255) & ~size_t(255); }

static EpLayout ep_layout(int P, int cap, int K, int H) {
  EpLayout L{};
  L.ready = 0;                       // u32 [4]: last published epoch of each buffer
  L.done = 64;                       // u32 [4][kEpMaxRanks]: epoch each reader has finished reading
  L.send_epoch = 256;                // u32 [4] (local)
  L.recv_epoch = 320;                // u32 [4] (local)
  L.counts = 512;                    // int [4][kEpMaxRanks]: rows per destination
  L.nent = 768;                      // int [kEpMaxRanks]: dispatch entries per destination
  size_t o = 1024;
  L.tcnt = o;  o += ep_al((size_t)((cap + kPlanTile - 1) / kPlanTile) * kEpMaxRanks * 2 * 4);  // int [tiles][P][2]
  const size_t rk = (size_t)P * cap * K;
  L.meta = o;  o += ep_al(rk * 4);   // int [P][cap][K]: local expert | k << 16, -1 after a row's entries
  L.wts = o;   o += ep_al(rk * 4);   // f32 [P][cap][K]: routing weight of each entry
  L.eoff = o;  o += ep_al((size_t)P * cap * 4);  // int [P][cap]: first entry of each row among the destination's
  L.dwts = o;  o += ep_al(rk * 4);   // f32 [P][cap][K]: backward return, d weight of each entry
  for (int b = 0; b < 4; ++b) {
    L.rows[b] = o;
    o += ep_al((size_t)P * cap * H * 2);  // bf16 [P][cap][H]
  }
  L.total = o;
  return L;
}

struct EpPeers {
  char* base[kEpMaxRanks];
};

// ------------------------------------------------------------------------------------------ flags
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// bounded wait until *p >= want (monotonic epoch); false after SMELB_WAIT_NS (status recorded)
__device__ bool ep_wait_ge(const uint32_t* p, uint32_t want, int* err, int who) {
  if (ld_acquire_sys(p) >= want) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t ns = 32;
  while (ld_acquire_sys(p) < want) {
    if (globaltimer_ns() - t0 > SMELB_WAIT_NS) {
      dev_fail_at(err, kDevErrEpWait, who, (int)want);
      return false;
    }
    __nanosleep(ns);
    ns = ns < 1024 ? 2 * ns : ns;
  }
  return true;
}

// sender: every reader (all ranks, itself included) has acknowledged the previous epoch of buffer b
__global__ void ep_wait_done_kernel(char* mine, EpLayout L, int P, int b, int* err) {
  const int d = threadIdx.x;
  if (d >= P) return;
  const uint32_t* done = reinterpret_cast<const uint32_t*>(mine + L.done) + b * kEpMaxRanks;
  const uint32_t want = reinterpret_cast<const uint32_t*>(mine + L.send_epoch)[b];
  ep_wait_ge(done + d, want, err, 100 * b + d);
}

// sender: the buffer's data (written by earlier kernels of the stream) is complete; publish the next epoch
__global__ void ep_publish_kernel(char* mine, EpLayout L, int b) {
  __threadfence_system();
  uint32_t* ep = reinterpret_cast<uint32_t*>(mine + L.send_epoch) + b;
  const uint32_t e = *ep + 1;
  *ep = e;
  st_release_sys(reinterpret_cast<uint32_t*>(mine + L.ready) + b, e);
}

// reader: every source has published the epoch this reader expects next
__global__ void ep_wait_ready_kernel(EpPeers peers, char* mine, EpLayout L, int P, int b, int* err) {
  const int s = threadIdx.x;
  if (s >= P) return;
  const uint32_t want = reinterpret_cast<const uint32_t*>(mine + L.recv_epoch)[b] + 1;
  ep_wait_ge(reinterpret_cast<const uint32_t*>(peers.base[s] + L.ready) + b, want, err, 1000 + 100 * b + s);
}

// reader: done reading every source's buffer b of this epoch
__global__ void ep_ack_kernel(EpPeers peers, char* mine, EpLayout L, int P, int rank, int b) {
  __shared__ uint32_t e;
  if (threadIdx.x == 0) e = reinterpret_cast<const uint32_t*>(mine + L.recv_epoch)[b] + 1;
  __syncthreads();
  __threadfence_system();
  const int s = threadIdx.x;
  if (s < P) st_release_sys(reinterpret_cast<uint32_t*>(peers.base[s] + L.done) + b * kEpMaxRanks + rank, e);
  __syncthreads();
  if (threadIdx.x == 0) reinterpret_cast<uint32_t*>(mine + L.recv_epoch)[b] = e;
}

// ------------------------------------------------------------------------------------------ block scan
// exclusive scan of (a, b) over the block (up to 1024 threads); returns the block totals in tot_a / tot_b
__device__ __forceinline__ void scan2(int a, int b, int& ex_a, int& ex_b, int& tot_a, int& tot_b) {
  __shared__ int wa[32], wb[32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int ia = a, ib = b;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int ta = __shfl_up_sync(0xffffffffu, ia, o), tb = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) {
      ia += ta;
      ib += tb;
    }
  }
  __syncthreads();  // wa / wb may still be read by the previous scan
  if (lane == 31) {
    wa[w] = ia;
    wb[w] = ib;
  }
  __syncthreads();
  if (w == 0) {
    int va = lane < (int)(blockDim.x >> 5) ? wa[lane] : 0, vb = lane < (int)(blockDim.x >> 5) ? wb[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int ta = __shfl_up_sync(0xffffffffu, va, o), tb = __shfl_up_sync(0xffffffffu, vb, o);
      if (lane >= o) {
        va += ta;
        vb += tb;
      }
    }
    wa[lane] = va;
    wb[lane] = vb;
  }
  __syncthreads();
  const int pa = w ? wa[w - 1] : 0, pb = w ? wb[w - 1] : 0;
  ex_a = pa + ia - a;
  ex_b = pb + ib - b;
  tot_a = wa[(blockDim.x >> 5) - 1];
  tot_b = wb[(blockDim.x >> 5) - 1];
}

// ------------------------------------------------------------------------------------------ source side
// The source-side plan, in token order (so the exchange is deterministic): for every destination d the tokens with
// at least one expert owned by d, their row position pos[t][d], the row's entries (local expert id and k, in k order)
// with their routing weights, the entry offset of every row and the slot j of every choice (t, k) within its row.
// Two passes over tiles of kPlanTile tokens: the tiles' row and entry counts per destination, then every tile writes
// its rows at the running offsets of the tiles before it.

// 5-bit count per destination of the token's choices it owns (K <= 16, P <= 8)
__device__ __forceinline__ unsigned long long plan_mask(const long long* __restrict__ topi,
                                                        const int* __restrict__ owner, int t, int T, int K) {
  unsigned long long m = 0;
  if (t >= T) return 0;
  long long e[kEpMaxK];
#pragma unroll
  for (int k = 0; k < kEpMaxK; ++k)
    if (k < K) e[k] = topi[(long long)t * K + k];
#pragma unroll
  for (int k = 0; k < kEpMaxK; ++k)
    if (k < K) m += 1ull << (5 * owner[e[k]]);
  return m;
}

__global__ void __launch_bounds__(kPlanTile) ep_plan_count_kernel(const long long* __restrict__ topi, int T, int K,
                                                                  const int* __restrict__ owner, int P, char* mine,
                                                                  EpLayout L) {
  __shared__ int part[kPlanTile / 32][kEpMaxRanks][2];
  const int t = blockIdx.x * kPlanTile + threadIdx.x, lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const unsigned long long m = plan_mask(topi, owner, t, T, K);
#pragma unroll
  for (int d = 0; d < kEpMaxRanks; ++d) {
    if (d >= P) break;
    const unsigned c = (unsigned)(m >> (5 * d)) & 31u;
    const unsigned r = __reduce_add_sync(0xffffffffu, c > 0 ? 1u : 0u), n = __reduce_add_sync(0xffffffffu, c);
    if (lane == 0) {
      part[w][d][0] = (int)r;
      part[w][d][1] = (int)n;
    }
  }
  __syncthreads();
  if (threadIdx.x < 2 * P) {
    const int d = threadIdx.x >> 1, q = threadIdx.x & 1;
    int v = 0;
    for (int i = 0; i < kPlanTile / 32; ++i) v += part[i][d][q];
    reinterpret_cast<int*>(mine + L.tcnt)[((long long)blockIdx.x * kEpMaxRanks + d) * 2 + q] = v;
  }
}

__global__ void __launch_bounds__(kPlanTile) ep_plan_fill_kernel(const long long* __restrict__ topi,
                                                                 const void* __restrict__ topv, int topv_f32, int T,
                                                                 int K, const int* __restrict__ owner,
                                                                 const int* __restrict__ local_id, int P, int cap,
                                                                 char* mine, EpLayout L, int* __restrict__ pos,
                                                                 int* __restrict__ slot_j, int* __restrict__ tok_of) {
  __shared__ int base[kEpMaxRanks][2];
  const int t = blockIdx.x * kPlanTile + threadIdx.x;
  const int* tcnt = reinterpret_cast<const int*>(mine + L.tcnt);
  if (threadIdx.x < 2 * P) {
    // running offsets of this tile per destination: the sums over the tiles before it (and, in the last tile, the
    // destination's totals)
    const int d = threadIdx.x >> 1, q = threadIdx.x & 1;
    int v = 0;
    for (int i = 0; i < (int)blockIdx.x; ++i) v += tcnt[((long long)i * kEpMaxRanks + d) * 2 + q];
    base[d][q] = v;
    if (blockIdx.x == gridDim.x - 1)
      reinterpret_cast<int*>(mine + (q ? L.nent : L.counts))[d] = v + tcnt[((long long)blockIdx.x * kEpMaxRanks + d) * 2 + q];
  }
  __syncthreads();
  const unsigned long long m = plan_mask(topi, owner, t, T, K);
  int* meta = reinterpret_cast<int*>(mine + L.meta);
  float* wts = reinterpret_cast<float*>(mine + L.wts);
  int* eoff = reinterpret_cast<int*>(mine + L.eoff);
  for (int d = 0; d < P; ++d) {
    const int c = (int)((m >> (5 * d)) & 31u);
    int pr, pe, tr, te;
    scan2(c > 0, c, pr, pe, tr, te);
    if (t >= T) continue;
    if (c == 0) {
      pos[(long long)t * P + d] = -1;
      continue;
    }
    const int p = base[d][0] + pr;
    const long long row = (long long)d * cap + p;
    tok_of[row] = t;
    pos[(long long)t * P + d] = p;
    eoff[row] = base[d][1] + pe;
    int j = 0;
    for (int k = 0; k < K; ++k) {
      const long long e = topi[(long long)t * K + k];
      if (owner[e] != d) continue;
      meta[row * K + j] = local_id[e] | (k << 16);
      wts[row * K + j] = topv_f32 ? reinterpret_cast<const float*>(topv)[(long long)t * K + k]
                                  : __bfloat162float(reinterpret_cast<const bf16*>(topv)[(long long)t * K + k]);
      slot_j[(long long)t * K + k] = j;
      ++j;
    }
    for (; j < K; ++j) meta[row * K + j] = -1;
  }
}

// One warp copies a row of vpr 16-byte vectors, each lane with up to 8 loads in flight before its stores (the source
// may be a peer's memory, where a load's latency is a few microseconds).
__device__ __forceinline__ void copy_row(uint4* __restrict__ dst, const uint4* __restrict__ src, int vpr, int lane) {
  for (int c0 = lane; c0 < vpr; c0 += 32 * 8) {
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (c0 + 32 * u < vpr) v[u] = src[c0 + 32 * u];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (c0 + 32 * u < vpr) dst[c0 + 32 * u] = v[u];
  }
}

// rows[b][d][i] = src[tok_of[d][i]] for the rows of every destination, one warp per row (16-byte copies);
// counts[b] = counts[0]
__global__ void ep_pack_rows_kernel(const bf16* __restrict__ src, int H, const int* __restrict__ tok_of, int P,
                                    int cap, char* mine, size_t counts_off, size_t rows_off, int b) {
  __shared__ int cnt[kEpMaxRanks];
  if (threadIdx.x < kEpMaxRanks) cnt[threadIdx.x] = threadIdx.x < P ? reinterpret_cast<const int*>(mine + counts_off)[threadIdx.x] : 0;
  __syncthreads();
  const int vpr = H / 8, lane = threadIdx.x & 31;
  const int nw = P * cap;
  uint4* dst = reinterpret_cast<uint4*>(mine + rows_off);
  for (int row = (int)((blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5); row < nw;
       row += (int)(((long long)gridDim.x * blockDim.x) >> 5)) {
    const int d = row / cap;
    if (row - d * cap >= cnt[d]) continue;
    copy_row(dst + (long long)row * vpr, reinterpret_cast<const uint4*>(src + (long long)tok_of[row] * H), vpr, lane);
  }
  if (b != 0 && blockIdx.x == 0 && threadIdx.x < P)
    reinterpret_cast<int*>(mine + counts_off)[b * kEpMaxRanks + threadIdx.x] = cnt[threadIdx.x];
}

// ------------------------------------------------------------------------------------------ owner side
// The rows every source s sent to this rank and their dispatch entries, numbered in (source, row, slot) order: entry n
// of row (s, i) slot j is base_s + eoff + j. Writes per entry its local expert (int64, the dispatch plan's input),
// source row (s * cap + i) and weight; per row its first entry and entry count; per source its row count. Blocks of
// 256 rows of one source (grid: row tiles x sources).
__global__ void __launch_bounds__(256) ep_recv_plan_kernel(EpPeers peers, EpLayout L, int P, int rank, int cap, int K,
                                                           long long cap_e, long long* __restrict__ entry_e,
                                                           int* __restrict__ entry_row, float* __restrict__ entry_w,
                                                           int* __restrict__ row_beg, int* __restrict__ row_m,
                                                           int* __restrict__ rc, int* __restrict__ n_total, int* err) {
  __shared__ long long s_base;
  __shared__ int s_c;
  const int s = blockIdx.y;
  const char* src = peers.base[s];
  if (threadIdx.x < 32) {
    // entries every source sends this rank (one remote read per source, in parallel over the lanes)
    const int q = threadIdx.x;
    const long long ne = q < P ? reinterpret_cast<const int*>(peers.base[q] + L.nent)[rank] : 0;
    long long before = q < s ? ne : 0, total = ne;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      before += __shfl_xor_sync(0xffffffffu, before, o);
      total += __shfl_xor_sync(0xffffffffu, total, o);
    }
    if (q == 0) {
      s_base = before;
      s_c = reinterpret_cast<const int*>(src + L.counts)[rank];
      if (blockIdx.x == 0) {
        rc[s] = s_c;
        if (s == 0) {
          *n_total = (int)(total < cap_e ? total : cap_e);
          if (total > cap_e) dev_fail_at(err, kDevErrEpCapacity, (int)total, (int)cap_e);
        }
      }
    }
  }
  __syncthreads();
  const int i = blockIdx.x * 256 + threadIdx.x;
  if (i >= s_c) return;
  const int* meta = reinterpret_cast<const int*>(src + L.meta) + ((long long)rank * cap + i) * K;
  const float* wts = reinterpret_cast<const float*>(src + L.wts) + ((long long)rank * cap + i) * K;
  const long long beg = s_base + reinterpret_cast<const int*>(src + L.eoff)[(long long)rank * cap + i];
  int mt[kEpMaxK];
  float wv[kEpMaxK];
#pragma unroll
  for (int j = 0; j < kEpMaxK; ++j)
    if (j < K) {
      mt[j] = meta[j];
      wv[j] = wts[j];
    }
  int m = 0;
#pragma unroll
  for (int j = 0; j < kEpMaxK; ++j) {
    if (j >= K || mt[j] < 0) break;
    const long long nn = beg + j;
    if (nn < cap_e) {
      entry_e[nn] = mt[j] & 0xFFFF;
      entry_row[nn] = s * cap + i;
      entry_w[nn] = wv[j];
    }
    ++m;
  }
  row_beg[(long long)s * cap + i] = (int)(beg < cap_e ? beg : cap_e);
  row_m[(long long)s * cap + i] = (int)(beg + m <= cap_e ? m : (beg < cap_e ? cap_e - beg : 0));  // kept entries
}

// entries past the received ones go to the sink expert, whose dispatch segment no GEMM reads
__global__ void ep_fill_sink_kernel(long long* __restrict__ entry_e, long long cap_e, const int* __restrict__ n_total,
                                    int sink) {
  const int n0 = *n_total;
  for (long long n = blockIdx.x * (long long)blockDim.x + threadIdx.x; n < cap_e; n += (long long)gridDim.x * blockDim.x)
    if (n >= n0) entry_e[n] = sink;
}

// local[s][i] = source s's rows[b][rank][i] for its rows (the one pull over NVLink per row and exchange), one warp per
// row; the row counts of the sources are read once per block
__global__ void ep_pull_rows_kernel(EpPeers peers, size_t counts_off, size_t rows_off, int P, int rank, int cap, int H,
                                    int b, bf16* __restrict__ local) {
  __shared__ int cnt[kEpMaxRanks];
  __shared__ const char* base[kEpMaxRanks];
  if (threadIdx.x < kEpMaxRanks) {
    const int s = threadIdx.x;
    base[s] = s < P ? peers.base[s] : nullptr;
    cnt[s] = s < P ? reinterpret_cast<const int*>(peers.base[s] + counts_off)[b * kEpMaxRanks + rank] : 0;
  }
  __syncthreads();
  const int vpr = H / 8, lane = threadIdx.x & 31;
  const int nw = P * cap;
  for (int row = (int)((blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5); row < nw;
       row += (int)(((long long)gridDim.x * blockDim.x) >> 5)) {
    const int s = row / cap, i = row - s * cap;
    if (i >= cnt[s]) continue;
    copy_row(reinterpret_cast<uint4*>(local) + (long long)row * vpr,
             reinterpret_cast<const uint4*>(base[s] + rows_off) + ((long long)rank * cap + i) * vpr, vpr, lane);
  }
}

// xs[row] = local[entry_row[src_of[row]]] for the dispatch rows before the sink segment (zeros on padding rows), one
// warp per row
__global__ void ep_gather_kernel(const bf16* __restrict__ local, const int* __restrict__ entry_row,
                                 const int* __restrict__ src_of, const int* __restrict__ offsets, int sink, int H,
                                 bf16* __restrict__ xs) {
  const int rows = offsets[sink];
  const int vpr = H / 8, lane = threadIdx.x & 31;
  for (int row = (int)((blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5); row < rows;
       row += (int)(((long long)gridDim.x * blockDim.x) >> 5)) {
    const int e = src_of[row];
    uint4* d4 = reinterpret_cast<uint4*>(xs) + (long long)row * vpr;
    if (e < 0) {
      for (int c = lane; c < vpr; c += 32) d4[c] = make_uint4(0, 0, 0, 0);
      continue;
    }
    copy_row(d4, reinterpret_cast<const uint4*>(local + (long long)entry_row[e] * H), vpr, lane);
  }
}

// One warp per received row (s, i): sum over its entries of w * y[row_of[entry]] (fp32, each product rounded before
// it is added, in slot order: the reference's y.float() * topv then sum, smel/moe.py:248-252) -> bf16 into this
// rank's rows[1][s][i]; counts[1][s] = rows received from s. Backward (bwd != 0): the entries' dX rows summed into
// rows[3] and each entry's d weight into dwts[s][i][j].
__global__ void ep_return_kernel(const bf16* __restrict__ y, const int* __restrict__ row_of,
                                 const float* __restrict__ entry_w, const float* __restrict__ entry_dw,
                                 const int* __restrict__ row_beg, const int* __restrict__ row_m, const int* __restrict__ rc,
                                 int P, int cap, int K, int H, char* mine, size_t counts_off, size_t rows_off,
                                 size_t dwts_off, int bwd) {
  const int b = bwd ? 3 : 1;
  const int lane = threadIdx.x & 31;
  const int nw = P * cap;
  bf16* out = reinterpret_cast<bf16*>(mine + rows_off);
  for (int wr = (int)((blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5); wr < nw;
       wr += (int)(((long long)gridDim.x * blockDim.x) >> 5)) {
    const int s = wr / cap, i = wr - s * cap;
    if (i >= rc[s]) continue;
    const int beg = row_beg[wr], m = row_m[wr];
    if (bwd && lane < m) reinterpret_cast<float*>(mine + dwts_off)[(long long)wr * K + lane] = entry_dw[beg + lane];
    // the row's entries, one per lane, broadcast below
    const int ro = lane < m ? row_of[beg + lane] : 0;
    const float wl = lane < m ? (bwd ? 1.0f : entry_w[beg + lane]) : 0.f;
    // four 256-column chunks per pass, each entry's four loads issued together
    for (int c0 = lane * 8; c0 < H; c0 += 1024) {
      float acc[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[u][q] = 0.f;
#pragma unroll 2
      for (int j = 0; j < m; ++j) {
        const float w = __shfl_sync(0xffffffffu, wl, j);
        const bf16* yr = y + (long long)__shfl_sync(0xffffffffu, ro, j) * H;
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (c0 + u * 256 < H) v[u] = *reinterpret_cast<const uint4*>(yr + c0 + u * 256);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (c0 + u * 256 >= H) break;
          const bf16* pv = reinterpret_cast<const bf16*>(&v[u]);
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[u][q] = __fadd_rn(acc[u][q], __fmul_rn(__bfloat162float(pv[q]), w));
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (c0 + u * 256 >= H) break;
        uint4 o;
        bf16* po = reinterpret_cast<bf16*>(&o);
#pragma unroll
        for (int q = 0; q < 8; ++q) po[q] = __float2bfloat16_rn(acc[u][q]);
        *reinterpret_cast<uint4*>(out + (long long)wr * H + c0 + u * 256) = o;
      }
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < P) reinterpret_cast<int*>(mine + counts_off)[b * kEpMaxRanks + threadIdx.x] =
                                              rc[threadIdx.x];
}

// One warp per dispatch row before the sink segment: dy[row] = bf16(g * w) of the entry's pulled gradient row and the
// entry's d weight sum_h g[h] * y[row][h] (fp32), the backward of the owner's share of smel/moe.py:248-252.
__global__ void ep_dy_kernel(const bf16* __restrict__ g_local, const int* __restrict__ entry_row,
                             const float* __restrict__ entry_w, const int* __restrict__ src_of,
                             const int* __restrict__ offsets, int sink, int H, const bf16* __restrict__ y,
                             bf16* __restrict__ dy, float* __restrict__ entry_dw) {
  const int rows = offsets[sink];
  const int lane = threadIdx.x & 31;
  for (long long row = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; row < rows;
       row += ((long long)gridDim.x * blockDim.x) >> 5) {
    const int e = src_of[row];
    float dot = 0.f;
    const float w = e >= 0 ? entry_w[e] : 0.f;
    const bf16* gr = e >= 0 ? g_local + (long long)entry_row[e] * H : nullptr;
    for (int c0 = lane * 8; c0 < H; c0 += 256) {
      uint4 o = make_uint4(0, 0, 0, 0);
      if (e >= 0) {
        const uint4 gv = *reinterpret_cast<const uint4*>(gr + c0);
        const uint4 yv = *reinterpret_cast<const uint4*>(y + row * H + c0);
        const bf16 *pg = reinterpret_cast<const bf16*>(&gv), *py = reinterpret_cast<const bf16*>(&yv);
        bf16* po = reinterpret_cast<bf16*>(&o);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float gf = __bfloat162float(pg[q]);
          po[q] = __float2bfloat16_rn(gf * w);
          dot = fmaf(gf, __bfloat162float(py[q]), dot);
        }
      }
      *reinterpret_cast<uint4*>(dy + row * H + c0) = o;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if (lane == 0 && e >= 0) entry_dw[e] = dot;
  }
}

// ------------------------------------------------------------------------------------------ source side, returns
// One warp per token: out[t] = bf16(sum over destinations d in rank order of the returned row rows[1 or 3][rank]
// [pos[t][d]] from d's region (fp32) + add[t]); backward also dtopv[t][k] = d's dwts[rank][pos][slot_j[t][k]].
__global__ void ep_collect_kernel(EpPeers peers, size_t rows_off, size_t dwts_off, int P, int rank, int cap, int K,
                                  int H, int T, const int* __restrict__ pos, const bf16* __restrict__ add,
                                  const bf16* __restrict__ gl, const float* __restrict__ dgl,
                                  const bf16* __restrict__ w_sg, int bwd,
                                  const long long* __restrict__ topi, const int* __restrict__ owner,
                                  const int* __restrict__ slot_j, void* __restrict__ dtopv, int dtopv_f32,
                                  bf16* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  for (int t = (int)((blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5); t < T;
       t += (int)(((long long)gridDim.x * blockDim.x) >> 5)) {
    // the token's partial row at every owner it was sent to (null where it was not)
    int pt[kEpMaxRanks];
    const bf16* rp[kEpMaxRanks];
#pragma unroll
    for (int d = 0; d < kEpMaxRanks; ++d) {
      pt[d] = d < P ? pos[(long long)t * P + d] : -1;
      rp[d] = pt[d] >= 0 ? reinterpret_cast<const bf16*>(peers.base[d] + rows_off) + ((long long)rank * cap + pt[d]) * H
                         : nullptr;
    }
    // the shared expert's gate of this token, rounded as the fused combine does
    const float sg = gl ? bf16_round(1.0f / (1.0f + expf(-__bfloat162float(gl[t])))) : 1.f;
    const float dg = dgl ? dgl[t] : 0.f;
    // per 256-column chunk every owner's load is issued before the sums (unrolled over the owners; owner order)
    for (int c0 = lane * 8; c0 < H; c0 += 256) {
      float acc[8];
      if (add) {
        const uint4 av = *reinterpret_cast<const uint4*>(add + (long long)t * H + c0);
        const bf16* pa = reinterpret_cast<const bf16*>(&av);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] = gl ? bf16_round(__bfloat162float(pa[q]) * sg) : __bfloat162float(pa[q]);
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] = 0.f;
      }
#pragma unroll
      for (int d = 0; d < kEpMaxRanks; ++d) {
        if (rp[d] == nullptr) continue;
        const uint4 v = *reinterpret_cast<const uint4*>(rp[d] + c0);
        const bf16* pv = reinterpret_cast<const bf16*>(&v);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(pv[q]);
      }
      if (dgl) {
        const uint4 wv = *reinterpret_cast<const uint4*>(w_sg + c0);
        const bf16* pw = reinterpret_cast<const bf16*>(&wv);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] = fmaf(dg, __bfloat162float(pw[q]), acc[q]);
      }
      uint4 o;
      bf16* po = reinterpret_cast<bf16*>(&o);
#pragma unroll
      for (int q = 0; q < 8; ++q) po[q] = __float2bfloat16_rn(acc[q]);
      *reinterpret_cast<uint4*>(out + (long long)t * H + c0) = o;
    }
    if (bwd && lane < K) {
      const int d = owner[topi[(long long)t * K + lane]];
      int p = 0;
      const char* base = nullptr;
#pragma unroll
      for (int dd = 0; dd < kEpMaxRanks; ++dd)
        if (dd == d) {
          p = pt[dd];
          base = peers.base[dd];
        }
      const float dw = reinterpret_cast<const float*>(base + dwts_off)[((long long)rank * cap + p) * K +
                                                                       slot_j[(long long)t * K + lane]];
      if (dtopv_f32) reinterpret_cast<float*>(dtopv)[(long long)t * K + lane] = dw;
      else reinterpret_cast<bf16*>(dtopv)[(long long)t * K + lane] = __float2bfloat16_rn(dw);
    }
  }
}

static int ep_grid(long long work, int threads) {
  return (int)std::min<long long>(std::max<long long>((work + threads - 1) / threads, 1), 148LL * 16);
}

static int ep_peers(const void* const* bases, int P, EpPeers& pr) {
  SMELB_CHECK_ARG(P >= 1 && P <= kEpMaxRanks, kErrShape, "ep: %d ranks (1..%d)", P, kEpMaxRanks);
  memset(&pr, 0, sizeof(pr));
  for (int s = 0; s < P; ++s) {
    SMELB_CHECK_ARG(bases[s] != nullptr, kErrArg, "ep: null region of rank %d", s);
    pr.base[s] = (char*)bases[s];
  }
  return kOk;
}

}  // namespace smelb

using namespace smelb;

// ================================================================================================== C ABI
extern "C" {

int64_t smelb_ep_region_bytes(int64_t P, int64_t cap, int64_t K, int64_t H) {
  // rows of all sources are indexed in 32 bits (P * cap), entries as P * cap * K
  if (P < 1 || P > kEpMaxRanks || cap < 1 || K < 1 || K > kEpMaxK || H < 8 || P * cap * K >= (1LL << 31)) return 0;
  return (int64_t)ep_layout((int)P, (int)cap, (int)K, (int)H).total;
}

int smelb_ep_region_alloc(int64_t bytes, void** region, void* ipc_handle) {
  SMELB_CHECK_ARG(region && ipc_handle && bytes > 0, kErrArg, "ep_region_alloc: bad arguments");
  void* p = nullptr;
  SMELB_CUDA(cudaMalloc(&p, (size_t)bytes));
  SMELB_CUDA(cudaMemset(p, 0, (size_t)bytes));
  cudaIpcMemHandle_t h;
  SMELB_CUDA(cudaIpcGetMemHandle(&h, p));
  memcpy(ipc_handle, &h, sizeof(h));
  *region = p;
  return kOk;
}

int smelb_ep_region_open(const void* ipc_handle, void** region) {
  SMELB_CHECK_ARG(region && ipc_handle, kErrArg, "ep_region_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  SMELB_CUDA(cudaIpcOpenMemHandle(region, h, cudaIpcMemLazyEnablePeerAccess));
  return kOk;
}

int smelb_ep_region_close(void* region) {
  SMELB_CUDA(cudaIpcCloseMemHandle(region));
  return kOk;
}

int smelb_ep_region_free(void* region) {
  SMELB_CUDA(cudaFree(region));
  return kOk;
}

int smelb_ep_sync(const void* const* regions, int64_t P, int64_t rank, int64_t cap, int64_t K, int64_t H, int op,
                  int buffer, void* stream) {
  EpPeers pr;
  const int rc = ep_peers(regions, (int)P, pr);
  if (rc != kOk) return rc;
  SMELB_CHECK_ARG(rank >= 0 && rank < P && buffer >= 0 && buffer < 4 && op >= 0 && op < 4, kErrArg,
                  "ep_sync: rank %lld buffer %d op %d", (long long)rank, buffer, op);
  int dev = 0;
  SMELB_CUDA(cudaGetDevice(&dev));
  int* err = device_status(dev);
  SMELB_CHECK_ARG(err != nullptr, kErrCuda, "ep_sync: no device status word");
  const EpLayout L = ep_layout((int)P, (int)cap, (int)K, (int)H);
  char* mine = pr.base[rank];
  cudaStream_t st = (cudaStream_t)stream;
  switch (op) {
    case SMELB_EP_WAIT_DONE: ep_wait_done_kernel<<<1, 32, 0, st>>>(mine, L, (int)P, buffer, err); break;
    case SMELB_EP_PUBLISH: ep_publish_kernel<<<1, 1, 0, st>>>(mine, L, buffer); break;
    case SMELB_EP_WAIT_READY: ep_wait_ready_kernel<<<1, 32, 0, st>>>(pr, mine, L, (int)P, buffer, err); break;
    default: ep_ack_kernel<<<1, 32, 0, st>>>(pr, mine, L, (int)P, (int)rank, buffer); break;
  }
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

int smelb_ep_plan(const int64_t* topi, const void* topv, int topv_fp32, int64_t T, int64_t K, const int32_t* owner,
                  const int32_t* local_id, const void* const* regions, int64_t P, int64_t rank, int64_t cap, int64_t H,
                  int32_t* pos, int32_t* slot_j, int32_t* tok_of, void* stream) {
  EpPeers pr;
  const int rc = ep_peers(regions, (int)P, pr);
  if (rc != kOk) return rc;
  SMELB_CHECK_ARG(topi && topv && owner && local_id && pos && slot_j && tok_of, kErrArg, "ep_plan: null pointer");
  SMELB_CHECK_ARG(T >= 0 && T <= cap && K >= 1 && K <= kEpMaxK && rank >= 0 && rank < P, kErrShape,
                  "ep_plan: T=%lld cap=%lld K=%lld", (long long)T, (long long)cap, (long long)K);
  const EpLayout L = ep_layout((int)P, (int)cap, (int)K, (int)H);
  const int tiles = (int)((T + kPlanTile - 1) / kPlanTile);
  cudaStream_t st = (cudaStream_t)stream;
  if (tiles == 0) {
    // no tokens: every destination gets zero rows and entries
    SMELB_CUDA(cudaMemsetAsync(pr.base[rank] + L.counts, 0, kEpMaxRanks * sizeof(int), st));
    SMELB_CUDA(cudaMemsetAsync(pr.base[rank] + L.nent, 0, kEpMaxRanks * sizeof(int), st));
    return kOk;
  }
  ep_plan_count_kernel<<<tiles, kPlanTile, 0, st>>>((const long long*)topi, (int)T, (int)K, owner, (int)P,
                                                    pr.base[rank], L);
  SMELB_CUDA(cudaGetLastError());
  ep_plan_fill_kernel<<<tiles, kPlanTile, 0, st>>>((const long long*)topi, topv, topv_fp32, (int)T, (int)K, owner,
                                                   local_id, (int)P, (int)cap, pr.base[rank], L, pos, slot_j, tok_of);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  count_launch();
  return kOk;
}

int smelb_ep_pack_rows(const void* src, int64_t H, const int32_t* tok_of, const void* const* regions, int64_t P,
                       int64_t rank, int64_t cap, int64_t K, int buffer, void* stream) {
  EpPeers pr;
  const int rc = ep_peers(regions, (int)P, pr);
  if (rc != kOk) return rc;
  SMELB_CHECK_ARG(src && tok_of && (buffer == 0 || buffer == 2) && H % 8 == 0, kErrArg, "ep_pack_rows: bad arguments");
  const EpLayout L = ep_layout((int)P, (int)cap, (int)K, (int)H);
  ep_pack_rows_kernel<<<ep_grid(P * cap * 32, 256), 256, 0, (cudaStream_t)stream>>>(
      (const bf16*)src, (int)H, tok_of, (int)P, (int)cap, pr.base[rank], L.counts, L.rows[buffer], buffer);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

int smelb_ep_recv_plan(const void* const* regions, int64_t P, int64_t rank, int64_t cap, int64_t K, int64_t H,
                       int64_t cap_entries, int64_t sink, int64_t* entry_e, int32_t* entry_row, float* entry_w,
                       int32_t* row_beg, int32_t* row_m, int32_t* recv_rows, int32_t* n_total, void* stream) {
  EpPeers pr;
  const int rc = ep_peers(regions, (int)P, pr);
  if (rc != kOk) return rc;
  SMELB_CHECK_ARG(entry_e && entry_row && entry_w && row_beg && row_m && recv_rows && n_total && cap_entries > 0,
                  kErrArg, "ep_recv_plan: bad arguments");
  int dev = 0;
  SMELB_CUDA(cudaGetDevice(&dev));
  int* err = device_status(dev);
  SMELB_CHECK_ARG(err != nullptr, kErrCuda, "ep_recv_plan: no device status word");
  const EpLayout L = ep_layout((int)P, (int)cap, (int)K, (int)H);
  cudaStream_t st = (cudaStream_t)stream;
  ep_recv_plan_kernel<<<dim3((unsigned)((cap + 255) / 256), (unsigned)P), 256, 0, st>>>(
      pr, L, (int)P, (int)rank, (int)cap, (int)K, cap_entries, (long long*)entry_e, entry_row, entry_w, row_beg, row_m,
      recv_rows, n_total, err);
  SMELB_CUDA(cudaGetLastError());
  ep_fill_sink_kernel<<<ep_grid(cap_entries, 256), 256, 0, st>>>((long long*)entry_e, cap_entries, n_total, (int)sink);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  count_launch();
  return kOk;
}

int smelb_ep_pull_rows(const void* const* regions, int64_t P, int64_t rank, int64_t cap, int64_t K, int64_t H,
                       int buffer, void* local, void* stream) {
  EpPeers pr;
  const int rc = ep_peers(regions, (int)P, pr);
  if (rc != kOk) return rc;
  SMELB_CHECK_ARG(local && (buffer == 0 || buffer == 2) && H % 8 == 0, kErrArg, "ep_pull_rows: bad arguments");
  const EpLayout L = ep_layout((int)P, (int)cap, (int)K, (int)H);
  ep_pull_rows_kernel<<<ep_grid(P * cap * 32, 256), 256, 0, (cudaStream_t)stream>>>(
      pr, L.counts, L.rows[buffer], (int)P, (int)rank, (int)cap, (int)H, buffer, (bf16*)local);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

int smelb_ep_gather(const void* local, const int32_t* entry_row, const int32_t* src_of, const int32_t* offsets,
                    int64_t sink, int64_t H, int64_t max_rows, void* xs, void* stream) {
  SMELB_CHECK_ARG(local && entry_row && src_of && offsets && xs && H % 8 == 0, kErrArg, "ep_gather: bad arguments");
  ep_gather_kernel<<<ep_grid(max_rows * 32, 256), 256, 0, (cudaStream_t)stream>>>(
      (const bf16*)local, entry_row, src_of, offsets, (int)sink, (int)H, (bf16*)xs);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

int smelb_ep_return(const void* y, const int32_t* row_of, const float* entry_w, const float* entry_dw,
                    const int32_t* row_beg, const int32_t* row_m, const int32_t* recv_rows, const void* const* regions,
                    int64_t P, int64_t rank, int64_t cap, int64_t K, int64_t H, int backward, void* stream) {
  EpPeers pr;
  const int rc = ep_peers(regions, (int)P, pr);
  if (rc != kOk) return rc;
  SMELB_CHECK_ARG(y && row_of && row_beg && row_m && recv_rows && (backward ? entry_dw != nullptr : entry_w != nullptr) &&
                      H % 256 == 0,
                  kErrArg, "ep_return: bad arguments (H a multiple of 256)");
  const EpLayout L = ep_layout((int)P, (int)cap, (int)K, (int)H);
  ep_return_kernel<<<ep_grid(P * cap * 32, 256), 256, 0, (cudaStream_t)stream>>>(
      (const bf16*)y, row_of, entry_w, entry_dw, row_beg, row_m, recv_rows, (int)P, (int)cap, (int)K, (int)H,
      pr.base[rank], L.counts, L.rows[backward ? 3 : 1], L.dwts, backward != 0);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

int smelb_ep_dy(const void* g_local, const int32_t* entry_row, const float* entry_w, const int32_t* src_of,
                const int32_t* offsets, int64_t sink, int64_t H, int64_t max_rows, const void* y, void* dy,
                float* entry_dw, void* stream) {
  SMELB_CHECK_ARG(g_local && entry_row && entry_w && src_of && offsets && y && dy && entry_dw && H % 256 == 0, kErrArg,
                  "ep_dy: bad arguments (H a multiple of 256)");
  ep_dy_kernel<<<ep_grid(max_rows * 32, 256), 256, 0, (cudaStream_t)stream>>>(
      (const bf16*)g_local, entry_row, entry_w, src_of, offsets, (int)sink, (int)H, (const bf16*)y, (bf16*)dy,
      entry_dw);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

int smelb_ep_collect(const void* const* regions, int64_t P, int64_t rank, int64_t cap, int64_t K, int64_t H, int64_t T,
                     const int32_t* pos, const void* add, const void* gate_logit, const float* dgl,
                     const void* w_sgate, int backward, const int64_t* topi, const int32_t* owner,
                     const int32_t* slot_j, void* dtopv, int dtopv_fp32, void* out, void* stream) {
  EpPeers pr;
  const int rc = ep_peers(regions, (int)P, pr);
  if (rc != kOk) return rc;
  SMELB_CHECK_ARG(pos && out && H % 256 == 0 && (!backward || (topi && owner && slot_j && dtopv)), kErrArg,
                  "ep_collect: bad arguments (H a multiple of 256)");
  SMELB_CHECK_ARG(!gate_logit || (add && !backward), kErrArg, "ep_collect: the gate applies to the forward's add");
  SMELB_CHECK_ARG(!dgl == !w_sgate && (!dgl || backward), kErrArg, "ep_collect: dgl and w_sgate go together");
  const EpLayout L = ep_layout((int)P, (int)cap, (int)K, (int)H);
  ep_collect_kernel<<<ep_grid(T * 32, 256), 256, 0, (cudaStream_t)stream>>>(
      pr, L.rows[backward ? 3 : 1], L.dwts, (int)P, (int)rank, (int)cap, (int)K, (int)H, (int)T, pos,
      (const bf16*)add, (const bf16*)gate_logit, dgl, (const bf16*)w_sgate, backward != 0,
      (const long long*)topi, owner, slot_j, dtopv, dtopv_fp32, (bf16*)out);
  SMELB_CUDA(cudaGetLastError());
  count_launch();
  return kOk;
}

}  // extern "C"
