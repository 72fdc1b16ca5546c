// Paged absorbed-MLA attention for B200 (sm_100a): scheduler, main tcgen05 kernel, combine.
//
// Numerics follow reference/src/tq_reference/mla_attention.py:135-169 with identity key
// absorption (q arrives absorbed) and value projection [I_512 | 0]: per query token and head,
//   s = (q . k) * scale,  p = exp(s - m) / sum(exp(s - m)),  out = sum p v,  lse = m + ln sum.
// Storage precision follows docs/TEST-PLAN.md:61-63 (f32 scores, f32 softmax, P rounded to bf16,
// f32 accumulation of P.V, output rounded once). A token with no visible key gets zeros and
// lse = -inf (mla_attention.py:147-148). The launch grid depends only on the device, never on the
// data (docs/TEST-PLAN.md:205-206); split-KV partial results merge by log-sum-exp.
//
// Kernel structure (one CTA pair = cluster of 2, one CTA per SM; rank r owns keys [32r, 32r+32)
// of every page for QK^T and value dims [256r, 256r+256) for PV and the output):
//   warp 0      TMA producer: the query's shared-memory slice per token, then per page this
//               CTA's 32 keys across all chunks and the peer's 32 keys across this CTA's value
//               chunks (3-stage ring, page-table entries read ahead); pages outside the pool are
//               fetched fully out of bounds (zeros) and flagged.
//   warp 1      MMA issuer (whole warp, one elected lane issues): S_r = Q K_r^T into TMEM
//               (M=128 heads, N=32 keys), then O_r += P V_r (M=128, N=256, K=16 keys per step)
//               with the own keys' P from TMEM and the peer keys' P from shared memory. It zeroes
//               the rows of a partial last page before the MMAs read them, so the NaN poison of
//               unused slots never reaches an accumulator.
//   warps 2-5   softmax and epilogue: one thread per head row (its TMEM lane). Per page: scores
//               to log2 units, mask, a candidate reference maximum (raised only when the page
//               maximum grows by more than 2^8; exact after the final normalisation), bf16
//               probabilities; the pair swaps probabilities and candidates through distributed
//               shared memory so both derive the same running maximum for their halves of O.
// Every wait is bounded (globaltimer); on timeout the CTA pair records TQ_DEV_WAIT_TIMEOUT,
// drains its in-flight TMA and MMA work, frees TMEM and exits.

#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <mutex>

#include "tq_contracts.h"
#include "tq_mla_layout.h"
#include "tq_ptx.cuh"

namespace tq {
namespace mla {

constexpr uint64_t kWaitTimeoutNs = 2000000000ull;   // 2 s: a wait this long means a fault
constexpr uint64_t kDrainTimeoutNs = 200000000ull;   // 0.2 s for draining in-flight copies
constexpr uint32_t kWaitMaxPolls = 1u << 22;          // second bound, independent of the timer
constexpr uint32_t kDrainMaxPolls = 1u << 20;
constexpr float kLn2 = 0.69314718055994530942f;
constexpr float kRescaleThreshold = 8.0f;            // log2 units

struct Meta {
  int* header;
  int* unit_n;
  int* unit_pages;
  int* unit_gstart;
  int* unit_first;
  int* unit_nsplit;
  int* unit_split_off;
  int* pair_begin;
  int* combine_list;
  int* empty_list;
  float* part_lse;
  float* part_out;
  int* sparse_rows;   // sparse plans: [T, topk] valid pool rows of each token, in entry order
  int* sparse_count;  // sparse plans: [T] valid entries (bits 0-23) and range flags (24-31)
  long long topk;     // 0 for dense plans
};

struct MainArgs {
  Meta meta;
  const char* q;
  long long q_stride_t;
  long long q_stride_h;
  const int* page_table;
  const int* seq_id;
  long long slots;
  long long pool_rows;
  int tokens;
  int heads;
  char* out;
  long long out_stride_t;
  long long out_stride_h;
  int out_f32;
  float* lse;
  float scale_log2;
  const uint8_t* kv;        // pool base (FP8 rows are read by the kernel's convert warps)
  long long kv_row_stride;  // bytes
};

// ---------------------------------------------------------------------------------------------
// Sparse plans: each token's valid index entries (j < k_len, 0 <= idx <= q_pos, idx < kv_len;
// docs/TEST-PLAN.md:199), in entry order, as pool rows page_table[s][idx / 64] * 64 + idx % 64.
// One block of 256 threads per token; thread i owns entries [9 i, 9 i + 9) (256 x 9 >= 2051), so
// all its index and page-table loads are in flight together, and one exclusive scan of the
// per-thread counts places every valid entry at its rank: the order does not depend on timing.
// An entry whose page lies outside the page table or the pool is dropped and flagged; invalid
// entries are never used to address the pool.

constexpr int kCompactPerThread = 9;
static_assert(TQ_MLA_MAX_TOPK <= 256 * kCompactPerThread, "index row exceeds one block's reach");

__global__ void __launch_bounds__(256) sparse_compact_kernel(
    Meta m, const int* __restrict__ idx, long long idx_stride, const int* __restrict__ k_len,
    const int* __restrict__ seq_id, const int* __restrict__ q_pos,
    const int* __restrict__ kv_len, const int* __restrict__ page_table, long long slots,
    long long pool_pages, int S, int T) {
  __shared__ int warp_n[8];
  __shared__ int block_flags;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    if (threadIdx.x == 0) block_flags = 0;
    const int s = seq_id[t];
    int flags = 0, mine = 0;
    int rows[kCompactPerThread];
    if (s < 0 || s >= S) {
      flags = TQ_DEV_SEQ_RANGE;
    } else {
      const long long kl = min((long long)k_len[t], m.topk);
      const int qp = q_pos[t], kvl = kv_len[s];
      const int* row_idx = idx + (long long)t * idx_stride;
      const int* pt = page_table + (long long)s * slots;
      const long long j0 = (long long)threadIdx.x * kCompactPerThread;
      int v[kCompactPerThread];
#pragma unroll
      for (int i = 0; i < kCompactPerThread; ++i) v[i] = j0 + i < kl ? row_idx[j0 + i] : -1;
#pragma unroll
      for (int i = 0; i < kCompactPerThread; ++i) {
        rows[i] = -1;
        if (v[i] >= 0 && v[i] <= qp && v[i] < kvl) {
          const long long pg = v[i] / kPageRows;
          if (pg >= slots) {
            flags |= TQ_DEV_TABLE_SHORT;
          } else {
            const int page = pt[pg];
            if (page < 0 || page >= pool_pages) flags |= TQ_DEV_PAGE_RANGE;
            else rows[i] = page * kPageRows + v[i] % kPageRows;
          }
        }
        mine += rows[i] >= 0;
      }
    }
    // Exclusive scan of the per-thread counts (entry order = thread order, then i).
    int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_n[w] = incl;
    flags = __reduce_or_sync(0xFFFFFFFFu, flags);
    __syncthreads();
    if (lane == 0 && flags) atomicOr(&block_flags, flags);
    int before = incl - mine, total = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      before += i < w ? warp_n[i] : 0;
      total += warp_n[i];
    }
    if (mine) {
      int* out = m.sparse_rows + (long long)t * m.topk + before;
#pragma unroll
      for (int i = 0; i < kCompactPerThread; ++i)
        if (rows[i] >= 0) *out++ = rows[i];
    }
    __syncthreads();
    if (threadIdx.x == 0) m.sparse_count[t] = total | (block_flags << 24);
    __syncthreads();  // warp_n and block_flags are reused by the next token
  }
}

// ---------------------------------------------------------------------------------------------
// Scheduler: one block of 1024 threads.

__device__ long long block_exclusive_scan(long long v, long long* total, long long* sh) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  long long x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    long long y = __shfl_up_sync(0xFFFFFFFFu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sh[w] = x;
  __syncthreads();
  if (w == 0) {
    long long t = sh[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      long long y = __shfl_up_sync(0xFFFFFFFFu, t, o);
      if (lane >= o) t += y;
    }
    sh[lane] = t;
  }
  __syncthreads();
  const long long before = w ? sh[w - 1] : 0;
  *total = sh[31];
  __syncthreads();
  return before + x - v;
}

__global__ void __launch_bounds__(1024) schedule_kernel(Meta m, const int* __restrict__ seq_id,
                                                        const int* __restrict__ q_pos,
                                                        const int* __restrict__ kv_len, int T,
                                                        int S, long long slots, long long pool_pages,
                                                        int pairs) {
  // Sparse plans: a token's keys are its valid index entries, counted by sparse_compact_kernel.
  __shared__ long long sh[32];
  __shared__ int s_err;
  ptx::grid_launch_dependents();  // the attention kernel may start its prologue meanwhile
  if (threadIdx.x == 0) s_err = 0;
  for (int c = threadIdx.x; c < pairs; c += blockDim.x) m.pair_begin[c] = -1;
  __syncthreads();
  const int per = (T + 1023) / 1024;
  const int lo = min(T, int(threadIdx.x) * per), hi = min(T, lo + per);

  // Units are laid end to end in a virtual page space: a unit with pages occupies
  // kSegmentCostPages (its start-up cost) followed by its pages; pair c takes the virtual range
  // [c * quota, (c + 1) * quota).
  long long my_vlen = 0;
  for (int u = lo; u < hi; ++u) {
    const int s = seq_id[u];
    long long n = 0;
    if (m.sparse_count) {
      const int v = m.sparse_count[u];
      n = v & 0xFFFFFF;
      if (v >> 24) atomicOr(&s_err, v >> 24);
    } else if (s < 0 || s >= S) {
      atomicOr(&s_err, TQ_DEV_SEQ_RANGE);
    } else {
      long long kl = kv_len[s];
      const long long cap = pool_pages > 0 ? slots * kPageRows : 0;
      if (kl > cap) {
        atomicOr(&s_err, pool_pages > 0 ? TQ_DEV_TABLE_SHORT : TQ_DEV_PAGE_RANGE);
        kl = cap;
      }
      n = min(kl, (long long)q_pos[u] + 1);
      if (n < 0) n = 0;
    }
    const int pages = int((n + kPageRows - 1) / kPageRows);
    m.unit_n[u] = int(n);
    m.unit_pages[u] = pages;
    my_vlen += pages > 0 ? pages + kSegmentCostPages : 0;
  }
  long long total = 0;
  long long g = block_exclusive_scan(my_vlen, &total, sh);
  if (total >= (1ll << 31)) {
    if (threadIdx.x == 0) atomicOr(&s_err, TQ_DEV_WORK_OVERFLOW);
    total = 0;
  }
  const long long quota = total ? (total + pairs - 1) / pairs : 0;
  long long my_split = 0;
  for (int u = lo; u < hi; ++u) {
    const int pages = total ? m.unit_pages[u] : 0;
    const long long a = g + (pages > 0 ? kSegmentCostPages : 0);  // virtual start of the pages
    m.unit_gstart[u] = int(a);
    int first = -1, ns = 0;
    if (pages > 0) {
      first = int(a / quota);
      ns = int((a + pages - 1) / quota) - first + 1;
      // Pairs whose range starts inside this unit's virtual span begin with it.
      const long long c_lo = (g + quota - 1) / quota, c_hi = (a + pages - 1) / quota;
      for (long long c = c_lo; c <= c_hi; ++c) m.pair_begin[c] = u;
    }
    m.unit_first[u] = first;
    m.unit_nsplit[u] = ns;
    my_split += ns >= 2 ? ns : 0;
    g = a + pages;
  }
  long long tmp;
  long long off = block_exclusive_scan(my_split, &tmp, sh);
  long long my_comb = 0, my_empty = 0;
  for (int u = lo; u < hi; ++u) {
    m.unit_split_off[u] = int(off);
    const int ns = m.unit_nsplit[u];
    off += ns >= 2 ? ns : 0;
    my_comb += ns >= 2;
    my_empty += (total ? m.unit_pages[u] : 0) == 0;
  }
  long long n_comb = 0, n_empty = 0;
  long long comb_at = block_exclusive_scan(my_comb, &n_comb, sh);
  long long empty_at = block_exclusive_scan(my_empty, &n_empty, sh);
  for (int u = lo; u < hi; ++u) {
    if (m.unit_nsplit[u] >= 2) m.combine_list[comb_at++] = u;
    if ((total ? m.unit_pages[u] : 0) == 0) m.empty_list[empty_at++] = u;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    m.header[kHdrError] = s_err;
    m.header[kHdrTotalPages] = int(total);
    m.header[kHdrQuota] = int(quota);
    m.header[kHdrNumCombine] = int(n_comb);
    m.header[kHdrNumEmpty] = int(n_empty);
    m.header[kHdrPairs] = pairs;
    m.header[kHdrTokens] = T;
    m.header[kHdrTimeoutWhere] = 0;
    m.header[kHdrTimeoutBar] = 0;
    m.header[kHdrTimeoutCta] = 0;
  }
}

// ---------------------------------------------------------------------------------------------
// Segment walk: the (token, first page, page count, partial slot) pieces a CTA pair processes.

struct Seg {
  int u, p0, np, slot;
};

struct SegWalker {
  long long g, g_end;  // virtual page positions
  int u, T, c;
  __device__ void init(const Meta& m, int pair, int tokens) {
    const long long total = m.header[kHdrTotalPages], quota = m.header[kHdrQuota];
    c = pair;
    T = tokens;
    g = g_end = 0;
    u = 0;
    if (quota == 0 || (long long)pair * quota >= total) return;
    u = m.pair_begin[pair];
    if (u < 0 || u >= tokens) return;  // no unit starts in this range, or bad metadata
    g = (long long)pair * quota;
    g_end = min(g + quota, total);
  }
  __device__ bool next(const Meta& m, Seg& s) {
    while (g < g_end && u < T) {
      const int pages = m.unit_pages[u];
      const long long a = m.unit_gstart[u], b = a + pages;
      if (pages <= 0 || g >= b) {
        ++u;
        continue;
      }
      if (g < a) g = a;  // skip the unit's start-up cost
      if (g >= g_end) return false;
      const int n = int(min(b, g_end) - g);
      s.u = u;
      s.p0 = int(g - a);
      s.np = n;
      const int ns = m.unit_nsplit[u];
      s.slot = ns >= 2 ? m.unit_split_off[u] + c - m.unit_first[u] : -1;
      g += n;
      ++u;
      return true;
    }
    return false;
  }
};

// ---------------------------------------------------------------------------------------------
// Bounded waits.

struct Waiter {
  volatile int* abort_flag;
  int* header;          // workspace header: error bits, then the first timeout's location
  uint32_t peer_abort;  // shared::cluster address of the peer's abort flag
  int where;            // caller role and page counter, recorded on timeout
  uint32_t bar_base;    // shared address of barrier 0

  __device__ void fail(uint32_t bar, uint32_t parity) {
    if (!*abort_flag) {
      *abort_flag = 1;
      ptx::st_cluster_u32(peer_abort, 1u);
      atomicOr(header + kHdrError, TQ_DEV_WAIT_TIMEOUT);
      if (atomicCAS(header + kHdrTimeoutWhere, 0, where | int(0x40000000)) == 0) {
        header[kHdrTimeoutBar] = int((bar - bar_base) / 8u) | int(parity << 16);
        header[kHdrTimeoutCta] = int(blockIdx.x) * 1024 + int(threadIdx.x);
      }
    }
  }

  // Bounded twice: by the global timer and by an iteration count, so a stalled timer cannot
  // turn a missed phase into an endless spin.
  template <bool kCluster>
  __device__ bool wait(uint32_t bar, uint32_t parity) {
    if (kCluster ? ptx::mbar_test_cluster(bar, parity) : ptx::mbar_test(bar, parity)) return true;
    const uint64_t t0 = ptx::global_timer_ns();
    for (uint32_t i = 1;; ++i) {
      if (kCluster ? ptx::mbar_test_cluster(bar, parity) : ptx::mbar_test(bar, parity))
        return true;
      if ((i & 63) == 0) {
        if (*abort_flag) return false;
        if (ptx::global_timer_ns() - t0 > kWaitTimeoutNs || i >= kWaitMaxPolls) {
          fail(bar, parity);
          return false;
        }
      }
    }
  }

  // Ignores the abort flag: used to drain work already in flight before the CTA exits.
  __device__ bool drain(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = ptx::global_timer_ns();
    for (uint32_t i = 1; !ptx::mbar_test(bar, parity); ++i) {
      if (ptx::global_timer_ns() - t0 > kDrainTimeoutNs || i >= kDrainMaxPolls) {
        fail(bar, parity);
        return false;
      }
    }
    return true;
  }
};

// ---------------------------------------------------------------------------------------------
// Main kernel.

// kFp8: FP8 E4M3 rows (512 codes, then 4 f32 scales, one per 128 values; no RoPE part).
// kSparse: a token's keys are its valid top-k index entries (the compacted pool rows of
// sparse_compact_kernel), 64 per page, instead of its sequence's positions.
// Either way four more warps (6-9) gather each page's rows and write the shared-memory operand
// layout the TMA gives dense bf16 rows, zeros past the token's keys: FP8 rows with plain loads
// and dequantization to bf16, sparse bf16 rows with cp.async. The MMA and softmax warps are
// unchanged.
template <bool kRope, bool kFp8 = false, bool kSparse = false>
__global__ void __launch_bounds__((kFp8 || kSparse) ? kThreadsGather : kThreads, 1)
    mla_paged_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_kv,
                     const __grid_constant__ CUtensorMap tm_v, const MainArgs a) {
  static_assert(!(kRope && kFp8), "FP8 rows carry no RoPE part");
  static_assert(!(kRope && kSparse), "sparse plans use 512-wide rows");
  constexpr bool kGather = kFp8 || kSparse;  // convert warps fill the pages' ring slots
  constexpr int kQkChunks = kRope ? 9 : 8;               // 64-dim chunks of the query width
  constexpr int kQSmemChunks = kQkChunks - kQTmemDims / 64;
  constexpr uint32_t kStageLoadBytes = (kQkChunks + 4) * kKvChunkBytes;
  constexpr uint32_t kOwnGroupBytes = kQkChunks * kAtomBytes;  // 8 own keys x all chunks
  constexpr uint32_t kPeerGroupBytes = 4 * kAtomBytes;         // 8 peer keys x value chunks
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = ptx::smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* sm = smem_raw + (base - raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = ptx::cluster_rank(), peer = rank ^ 1u;
  const int pair = int(ptx::cluster_id_x());
  auto bar = [&](int i) -> uint32_t { return base + kSmBars + 8u * uint32_t(i); };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + kSmMisc + 4);
  const uint32_t* tmem_holder = reinterpret_cast<const uint32_t*>(sm + kSmMisc);
  Waiter wt{abort_flag, a.meta.header, ptx::map_peer(base + kSmMisc + 4, peer), 0,
            base + kSmBars};

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      // FP8 / sparse: a page's stage is complete when the four convert warps have arrived (FP8:
      // each arrival also expects the peer's 4 KB copy of its keys' value half); a query slot's
      // TMA arrives once with its bytes plus three plain arrivals.
      ptx::mbar_init(bar(kBarKvFull + s), kGather ? kConvertWarps : 1);
      ptx::mbar_init(bar(kBarKvEmpty + s), 1);
      ptx::mbar_init(bar(kBarKvGrant + s), 1);
      ptx::mbar_init(bar(kBarPeerGrant + s), 1);
    }
    ptx::mbar_init(bar(kBarQSmemFull), 1);
    ptx::mbar_init(bar(kBarQEmpty), 1);
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(bar(kBarSFull + b), 1);
      ptx::mbar_init(bar(kBarPFull + b), kSoftmaxWarps);
      ptx::mbar_init(bar(kBarPvDone + b), 1);
    }
    ptx::mbar_init(bar(kBarOFull), 1);
    ptx::mbar_init(bar(kBarOFree), kSoftmaxWarps);
    for (int i = 0; i < 2; ++i) ptx::mbar_init(bar(kBarMsgFree + i), 1);
    for (int i = 0; i < 8; ++i) {
      ptx::mbar_init(bar(kBarMsgFull + i), 1);
      // Each receive buffer expects one peer warp's message; armed for pages 0 and 1.
      ptx::mbar_expect_tx(bar(kBarMsgFull + i), kWarpMsgBytes);
    }
    for (int w = 0; w < 4; ++w) {
      ptx::mbar_init(bar(kBarLsumFull + w), 1);
      ptx::mbar_expect_tx(bar(kBarLsumFull + w), 32 * 4);
    }
    ptx::mbar_init(bar(kBarDrain), 1);
    *abort_flag = 0;
    ptx::fence_mbar_init_cluster();
    ptx::tma_prefetch_desc(&tm_q);
    ptx::tma_prefetch_desc(&tm_kv);
    ptx::tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    ptx::tmem_alloc(base + kSmMisc, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  // Everything above overlaps the scheduler kernel; its outputs are read from here on. The
  // combine grid may then launch early and wait for this grid in turn.
  ptx::grid_dependency_wait();
  ptx::grid_launch_dependents();
  SegWalker walker;
  walker.init(a.meta, pair, a.tokens);
  const Meta& meta = a.meta;
  const int key0 = kKeysPerCta * int(rank);  // this CTA's keys within a page
  const int vdim0 = kValueHalf * int(rank);  // this CTA's value dims

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t it = 0, useq = 0;
      Seg s;
      bool ok = true;
      // A sequence with one query token has its KV rows read once per launch (by this pair,
      // within a page's time): evict-first keeps them from displacing the page tables, queries
      // and split partials in L2. Rows of a sequence with several query tokens (multi-token
      // decode, prefill chunks; adjacent tokens) are read again and keep the normal priority.
      const uint64_t policy_once = ptx::l2_policy_evict_first();
      const uint64_t policy_reused = ptx::l2_policy_evict_normal();
      while (ok && walker.next(meta, s)) {
        const int sq = a.seq_id[s.u];
        const bool reused = (s.u > 0 && a.seq_id[s.u - 1] == sq) ||
                            (s.u + 1 < a.tokens && a.seq_id[s.u + 1] == sq);
        const uint64_t kv_policy = reused ? policy_reused : policy_once;
        // Page-table entries are read three pages ahead of their loads: a dependent global read
        // at load time would add its latency to every page's arrival.
        const int* pt = a.page_table + (long long)sq * a.slots;
        int pf0 = (!kGather && s.np > 0) ? pt[s.p0] : 0;
        int pf1 = (!kGather && s.np > 1) ? pt[s.p0 + 1] : 0;
        int pf2 = (!kGather && s.np > 2) ? pt[s.p0 + 2] : 0;
        // Query dims [0, 384) pass through two ring slots, three 64-dim chunks each, on their way
        // to TMEM (tcgen05.cp by the MMA warp). The query boxes are 128 rows high: rows past the
        // head count lie outside the tensor and arrive as zeros.
        for (int qp = 0; qp < 2; ++qp, ++it) {
          const uint32_t stage = it % kStages;
          wt.where = (1 << 24) | int(it & 0xFFFFFF);
          if (!wt.wait<false>(bar(kBarKvEmpty + stage), ((it / kStages) & 1u) ^ 1u)) {
            ok = false;
            break;
          }
          const uint32_t fb = bar(kBarKvFull + stage);
          ptx::mbar_expect_tx(fb, 3 * kQChunkBytes);
          if constexpr (kGather) {
            for (int k = 1; k < kConvertWarps; ++k) ptx::mbar_arrive(fb);
          }
          for (int k = 0; k < 3; ++k)
            ptx::tma_load_3d(base + kSmKv + stage * kStageBytes + k * kQChunkBytes, &tm_q, fb,
                             64 * (3 * qp + k), 0, s.u);
        }
        if (!ok) break;
        wt.where = (1 << 24) | int(it & 0xFFFFFF);
        if (!wt.wait<false>(bar(kBarQEmpty), (useq & 1u) ^ 1u)) break;
        ptx::mbar_expect_tx(bar(kBarQSmemFull), kQChunkBytes * kQSmemChunks);
        for (int k = 0; k < kQSmemChunks; ++k)
          ptx::tma_load_3d(base + kSmQ + k * kQChunkBytes, &tm_q, bar(kBarQSmemFull),
                           kQTmemDims + 64 * k, 0, s.u);
        ++useq;
        // FP8 / sparse: the convert warps fill the pages' stages; this loop waits for each page's slot
        // to be free and grants it to them. This thread is the only waiter on kBarKvEmpty and
        // waits on every slot in ring order: a parity wait tells completions apart only modulo
        // 2, so a waiter that skipped slots could pass two phases early or block one phase late.
        // A stage's grants are at most one ahead of the convert warps (the next grant on it
        // needs the previous page's release), so their waits on kBarKvGrant are exact.
        for (int j = 0; j < s.np; ++j, ++it) {
          const uint32_t stage = it % kStages;
          const int page = pf0;
          pf0 = pf1;
          pf1 = pf2;
          pf2 = (!kGather && j + 3 < s.np) ? pt[s.p0 + j + 3] : 0;
          wt.where = (1 << 24) | int(it & 0xFFFFFF);
          if (!wt.wait<false>(bar(kBarKvEmpty + stage), ((it / kStages) & 1u) ^ 1u)) {
            ok = false;
            break;
          }
          if constexpr (kGather) {
            ptx::mbar_arrive(bar(kBarKvGrant + stage));
            // FP8: the peer's convert warps may now copy their keys' value half into this stage.
            if constexpr (kFp8) ptx::mbar_arrive_cluster(ptx::map_peer(bar(kBarPeerGrant + stage), peer));
            continue;
          }
          long long row = (long long)page * kPageRows;
          if (page < 0 || row >= a.pool_rows) {
            atomicOr(a.meta.header + kHdrError, TQ_DEV_PAGE_RANGE);
            row = a.pool_rows;  // a box entirely out of bounds: TMA fills zeros
          }
          const uint32_t dst = base + kSmKv + stage * kStageBytes;
          const uint32_t fb = bar(kBarKvFull + stage);
          // Two requests per stage (the TMA unit's cost is largely per request): this CTA's keys
          // across every 64-dim chunk, then the peer's keys across this CTA's value chunks. The
          // map's axes are {64 dims, key in group, chunk, 8-key group}: a box reads each 8-row
          // group's contiguous bytes in one go and lands as [group][chunk][8 keys x 128 B].
          ptx::mbar_expect_tx(fb, kStageLoadBytes);
          ptx::tma_load_4d_hint(dst, &tm_kv, fb, 0, 0, 0, int((row + key0) / 8), kv_policy);
          ptx::tma_load_4d_hint(dst + kPvxOffset, &tm_v, fb, 0, 0, vdim0 / 64,
                                int((row + kKeysPerCta - key0) / 8), kv_policy);
        }
      }
      // Drain: every issued copy has landed before the CTA may exit.
      for (uint32_t st = 0; st < kStages && st < it; ++st) {
        const uint32_t last = it - 1 - ((it - 1 - st) % kStages);
        wt.drain(bar(kBarKvFull + st), (last / kStages) & 1u);
      }
      if (useq) wt.drain(bar(kBarQSmemFull), (useq - 1) & 1u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // QK^T: S[128 x 32] = Q x K_own^T, 24 steps with the query from TMEM, then the remaining
    // query chunks from shared memory. PV: O_half[128 x 256] += P[128 x 64] V[64 x 256]: the
    // own keys' P from TMEM (aliased over the scores), the peer keys' P from shared memory.
    // Issue order per step j (QK(j) already issued and its S(j) committed, so the softmax of
    // page j runs while the pipe works): wait for P(j-1); PV(j-1) and its commits; wait for page
    // j+1's data; QK(j+1) and the commit of S(j+1). Queued back to back, PV(j-1) and QK(j+1)
    // interleave in the pipe and PV's stage release comes late (measured slower); with the data
    // wait between them, PV(j-1) drains first and frees its KV stage for the producer sooner.
    // S buffer j%2 is rewritten by QK(j+2) only after PV(j) was issued: the pipe executes in
    // issue order, so P(j) is read before it is overwritten.
    // The whole warp runs this loop converged: waits are made warp-uniform, and each MMA and
    // commit is issued by one lane elected inside the instruction sequence.
    constexpr uint32_t idesc_qk = ptx::idesc_bf16(128, 32, 0);
    constexpr uint32_t idesc_pv = ptx::idesc_bf16(128, 256, 1);
    uint32_t it = 0, useq = 0;
    Seg s;
    bool ok = true;
    auto wait_all = [&](uint32_t b, uint32_t parity) -> bool {
      const bool r = wt.wait<false>(b, parity);
      return __all_sync(0xFFFFFFFFu, r);
    };
    // Waits for page itq (page `p` of its sequence, `n` visible keys) and zeroes its rows past
    // the cached length (NaN-poisoned slots) before any MMA reads them.
    auto prepare = [&](uint32_t rq, int p, int n) -> bool {
      const uint32_t stage = rq % kStages;
      if (!wait_all(bar(kBarKvFull + stage), (rq / kStages) & 1u)) return false;
      const int valid = min(kPageRows, n - p * kPageRows);
      const int own_valid = max(0, min(kKeysPerCta, valid - key0));
      const int peer_valid = max(0, min(kKeysPerCta, valid - (kKeysPerCta - key0)));
      // FP8 / sparse: the convert warps already wrote zeros past the token's keys.
      if (!kGather && (own_valid < kKeysPerCta || peer_valid < kKeysPerCta)) {
        uint8_t* st_ptr = sm + kSmKv + stage * kStageBytes;
        const int own_words = (kKeysPerCta - own_valid) * 8;
        const int peer_words = (kKeysPerCta - peer_valid) * 8;
        // Key r of chunk c sits at (r / 8) * group bytes + c * 1 KB + (r % 8) * 128 B.
        for (int i = lane; i < kQkChunks * own_words; i += 32) {
          const int c = i / own_words, r = own_valid + (i % own_words) / 8, w = i % 8;
          reinterpret_cast<uint4*>(st_ptr + (r >> 3) * kOwnGroupBytes + c * kAtomBytes +
                                   (r & 7) * 128)[w] = make_uint4(0, 0, 0, 0);
        }
        for (int i = lane; i < 4 * peer_words; i += 32) {
          const int c = i / peer_words, r = peer_valid + (i % peer_words) / 8, w = i % 8;
          reinterpret_cast<uint4*>(st_ptr + kPvxOffset + (r >> 3) * kPeerGroupBytes +
                                   c * kAtomBytes + (r & 7) * 128)[w] = make_uint4(0, 0, 0, 0);
        }
        ptx::fence_proxy_async_smem();
        __syncwarp();
      }
      return true;
    };
    // Descriptors advance by compile-time offsets (start field = address >> 4; shared addresses
    // stay below 256 KB, so the 14-bit field never carries).
    auto issue_qk = [&](uint32_t itq, uint32_t rq) {
      const uint32_t stage_base = base + kSmKv + (rq % kStages) * kStageBytes;
      const uint32_t d = tmem + kTmemS + (itq & 1u) * 32;
      // K-major, 128B swizzle: 8-key groups kOwnGroupBytes apart, chunks 1 KB apart.
      const uint64_t kd = ptx::smem_desc(stage_base, 16, kOwnGroupBytes, 2);
      const uint64_t qd = ptx::smem_desc(base + kSmQ, 16, 1024, 2);
#pragma unroll
      for (int kk = 0; kk < kQTmemDims / 16; ++kk)
        ptx::mma_ts_warp(d, tmem + kTmemQ + kk * 8,
                         kd + uint64_t(((kk >> 2) * kAtomBytes + (kk & 3) * 32) >> 4),
                         idesc_qk, kk != 0);
#pragma unroll
      for (int kk = 0; kk < kQSmemChunks * 4; ++kk)
        ptx::mma_ss_warp(d, qd + uint64_t(((kk >> 2) * kQChunkBytes + (kk & 3) * 32) >> 4),
                         kd + uint64_t((((kQTmemDims / 64) + (kk >> 2)) * kAtomBytes +
                                        (kk & 3) * 32) >> 4),
                         idesc_qk, 1);
    };
    auto issue_pv = [&](uint32_t itp, uint32_t rp, bool first) {
      const uint32_t stage = rp % kStages, pb = itp & 1u;
      const uint32_t stage_base = base + kSmKv + stage * kStageBytes;
      // V as B, MN-major: 64-dim chunks 1 KB apart (LBO), 8-key groups one group apart (SBO).
      const uint64_t vd =
          ptx::smem_desc(stage_base + (vdim0 / 64) * kAtomBytes, kAtomBytes, kOwnGroupBytes, 2);
      const uint64_t xd =
          ptx::smem_desc(stage_base + kPvxOffset, kAtomBytes, kPeerGroupBytes, 2);
      // Peer P, K-major without swizzle: 8-row groups 128 B apart (SBO), the two 8-key chunks of
      // a step 2 KB apart (LBO).
      const uint64_t pd = ptx::smem_desc(base + kSmPeer + pb * kPMsgBytes, kPChunkBytes, 128, 0);
#pragma unroll
      for (int kk = 0; kk < 2; ++kk)
        ptx::mma_ts_warp(tmem + kTmemO, tmem + kTmemS + pb * 32 + kk * 8,
                         vd + uint64_t((kk * 2 * kOwnGroupBytes) >> 4), idesc_pv,
                         (!first || kk > 0) ? 1u : 0u);
#pragma unroll
      for (int kk = 0; kk < 2; ++kk)
        ptx::mma_ss_warp(tmem + kTmemO, pd + uint64_t((kk * 2 * kPChunkBytes) >> 4),
                         xd + uint64_t((kk * 2 * kPeerGroupBytes) >> 4), idesc_pv, 1u);
      ptx::mma_commit_warp(bar(kBarKvEmpty + stage));
      ptx::mma_commit_warp(bar(kBarPvDone + pb));
      // The peer's message buffer pb in this CTA is consumed: the peer may write its next one.
      ptx::mma_commit_multicast_warp(bar(kBarMsgFree + pb), uint16_t(1u << peer));
    };
    uint32_t ring = 0;  // ring slots consumed: two query slots per segment, then its pages
    while (ok && walker.next(meta, s)) {
      const int n = meta.unit_n[s.u];
      const uint32_t it0 = it;
      wt.where = (2 << 24) | int(it0 & 0xFFFFFF);
      // Query dims [0, 384) into TMEM from the two query slots, once the previous segment's QK
      // MMAs (the readers of the old query) have completed. The copies and the MMAs after them
      // run in issue order; each slot is released when its copies are done.
      if (useq > 0 && !wait_all(bar(kBarQEmpty), (useq - 1) & 1u)) break;
      for (int qp = 0; qp < 2 && ok; ++qp) {
        const uint32_t rq = ring + qp, stage = rq % kStages;
        if (!wait_all(bar(kBarKvFull + stage), (rq / kStages) & 1u)) { ok = false; break; }
        ptx::tc_fence_after();
        const uint32_t src = base + kSmKv + stage * kStageBytes;
#pragma unroll
        for (int c = 0; c < 12; ++c)
          ptx::cp_smem_to_tmem_warp(
              tmem + kTmemQ + (qp * 12 + c) * 8,
              ptx::smem_desc(src + (c >> 2) * kQChunkBytes + (c & 3) * 32, 16, 1024, 2));
        ptx::mma_commit_warp(bar(kBarKvEmpty + stage));
      }
      if (!ok) break;
      const uint32_t r0 = ring + 2;  // ring slot of the segment's first page
      if (!wait_all(bar(kBarQSmemFull), useq & 1u)) break;
      if (!prepare(r0, s.p0, n)) break;
      ptx::tc_fence_after();
      issue_qk(it0, r0);
      ptx::mma_commit_warp(bar(kBarSFull + (it0 & 1u)));
      if (s.np == 1) ptx::mma_commit_warp(bar(kBarQEmpty));
      for (int j = 0; j < s.np; ++j) {
        const uint32_t itq = it0 + j;  // QK(itq) is issued and committed
        const bool has_next = j + 1 < s.np;
        wt.where = (2 << 24) | int(itq & 0xFFFFFF);
        if (j >= 1) {
          const uint32_t itp = itq - 1;
          if (j == 1 && !wait_all(bar(kBarOFree), (useq & 1u) ^ 1u)) { ok = false; break; }
          if (!wait_all(bar(kBarPFull + (itp & 1u)), (itp >> 1) & 1u)) { ok = false; break; }
          ptx::tc_fence_after();
          issue_pv(itp, r0 + j - 1, j == 1);
        }
        // Waiting here, after PV(j-1) was issued, keeps QK(j+1) out of the pipe until page j+1's
        // data is in, which in practice lets PV(j-1) drain first and release its KV stage early.
        if (has_next && !prepare(r0 + j + 1, s.p0 + j + 1, n)) { ok = false; break; }
        ptx::tc_fence_after();
        if (has_next) {
          issue_qk(itq + 1, r0 + j + 1);
          ptx::mma_commit_warp(bar(kBarSFull + ((itq + 1) & 1u)));
          if (j + 2 == s.np) ptx::mma_commit_warp(bar(kBarQEmpty));
        }
        __syncwarp();
      }
      if (!ok) break;
      // PV of the segment's last page completes this token's output.
      const uint32_t itp = it0 + s.np - 1;
      wt.where = (2 << 24) | int(itp & 0xFFFFFF);
      if (s.np == 1 && !wait_all(bar(kBarOFree), (useq & 1u) ^ 1u)) { ok = false; break; }
      if (!wait_all(bar(kBarPFull + (itp & 1u)), (itp >> 1) & 1u)) { ok = false; break; }
      ptx::tc_fence_after();
      issue_pv(itp, r0 + s.np - 1, s.np == 1);
      ptx::mma_commit_warp(bar(kBarOFull));
      __syncwarp();
      it = it0 + s.np;
      ring = r0 + s.np;
      ++useq;
    }
    if (lane == 0) ptx::mma_commit(bar(kBarDrain));
    __syncwarp();
    wt.drain(bar(kBarDrain), 0);
  } else if (warp >= 6) {
    // ------------------------------------------------------------------ convert warps
    // Warp cw handles this CTA's keys key0 + 8 cw + [0, 8) across all 512 dims (lane: dims
    // [16 lane, 16 lane + 16)) and the peer's keys (32 - key0) + 8 cw + [0, 8) across this CTA's
    // 256 value dims (two keys per instruction, 16 lanes each). Each lane's 16 dims are two bf16
    // 16-byte units, written at their 128B-swizzled places (unit u of row r at u ^ (r % 8)).
    // Keys past the token's count (and rows of pages outside the pool) are written as zeros and
    // their rows are never read. A page's pool rows: page_table[seq][p] * 64 + key (dense), or
    // the token's compacted valid entries p * 64 + key (sparse).
    // FP8 rows: each 16-byte group of codes is dequantized (code x tile scale, rounded once to
    // bf16) and stored. Sparse bf16 rows: cp.async copies straight into the stage after the
    // grant, zero-filled past the count.
    if constexpr (kFp8) {
      // FP8 rows. Warp cw converts this CTA's keys key0 + 8 cw + [0, 8) across all 512 dims (lane:
      // dims [16 lane, 16 lane + 16)) into its own group of the page's stage, then copies the
      // group's four 64-dim chunks of the peer's value half (4 KB, already in the peer's layout)
      // into the peer's stage with one bulk copy, once the peer's producer has granted that stage
      // (kBarPeerGrant); the peer does the same for its keys, so each key is loaded and converted
      // once per pair. Each warp's arrival on its own stage expects the peer's 4 KB.
      // The next page's codes (cp.async, zero-filled past the token's keys or outside the pool)
      // are copied into a per-warp buffer in the unused query chunk once this page's conversion
      // has read it, and land while the pair works through the grants and copies: 8 keys x
      // four 128-code tiles (tile t of key i at t KB + i * 128 B), scale quadruples at
      // kSmFp8Scales. The page-table entry (dense) or the 8 row numbers (sparse) of the page after
      // next are read one page ahead.
      static_assert(kQSmemChunks + 1 <= int(kSmKv / kQChunkBytes), "no free query chunk for FP8 codes");
      const int cw = warp - 6;
      const uint32_t raw = base + kSmQ + kQSmemChunks * kQChunkBytes + cw * 4096;
      const uint8_t* raw_p = sm + kSmQ + kQSmemChunks * kQChunkBytes + cw * 4096;
      const uint32_t rsc = base + kSmFp8Scales + cw * 128;
      const uint8_t* rsc_p = sm + kSmFp8Scales + cw * 128;
      const uint32_t peer_chunk0 = uint32_t((kValueHalf - vdim0) / 64);  // the peer's value chunks
      uint32_t it = 0;
      uint32_t grant_parity = 0, peer_parity = 0;  // bit s: parity of stage s's next phase
      Seg s;
      bool ok = true;
      while (ok && walker.next(meta, s)) {
        const int n = meta.unit_n[s.u];
        const int* pt = kSparse ? nullptr : a.page_table + (long long)a.seq_id[s.u] * a.slots;
        const int* srows = kSparse ? meta.sparse_rows + (long long)s.u * meta.topk : nullptr;
        // Row numbers of page p's 8 keys of this warp (-1: zero-filled), from `ent`: the page-table
        // entry (dense, in ent[0]) or the 8 compacted rows (sparse).
        auto fetch = [&](int p, int (&ent)[8]) {
          const int valid = min(kPageRows, n - p * kPageRows);
          if constexpr (kSparse) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int key = key0 + 8 * cw + i;
              ent[i] = key < valid ? srows[p * kPageRows + key] : -1;
            }
          } else {
            ent[0] = pt[p];
          }
        };
        auto issue = [&](int p, const int (&ent)[8]) {
          const int valid = min(kPageRows, n - p * kPageRows);
          long long row0 = 0;
          bool page_ok = true;
          if constexpr (!kSparse) {
            row0 = (long long)ent[0] * kPageRows;
            page_ok = ent[0] >= 0 && row0 < a.pool_rows;
            if (!page_ok && cw == 0 && lane == 0)
              atomicOr(a.meta.header + kHdrError, TQ_DEV_PAGE_RANGE);
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int key = key0 + 8 * cw + i;
            bool live;
            long long row;
            if constexpr (kSparse) {
              live = ent[i] >= 0;
              row = ent[i];
            } else {
              live = page_ok && key < valid;
              row = row0 + key;
            }
            const uint8_t* rp = live ? a.kv + row * a.kv_row_stride : a.kv;
            ptx::cp_async_16(raw + (lane >> 3) * kAtomBytes + i * 128 + (lane & 7) * 16,
                             rp + (live ? 16 * lane : 0), live ? 16u : 0u);
            if (lane == i)
              ptx::cp_async_16(rsc + i * 16, rp + (live ? kFp8RowCodes : 0), live ? 16u : 0u);
          }
          ptx::cp_async_commit();
        };
        it += 2;  // the segment's two query slots, filled by the TMA producer
        int ent[8], nxt[8];
        fetch(s.p0, ent);
        issue(s.p0, ent);
        if (s.np > 1) fetch(s.p0 + 1, nxt);
        for (int j = 0; j < s.np; ++j, ++it) {
          const uint32_t stage = it % kStages;
          wt.where = (7 << 24) | int(it & 0xFFFFFF);
          const bool got =
              wt.wait<false>(bar(kBarKvGrant + stage), (grant_parity >> stage) & 1u);
          if (!__all_sync(0xFFFFFFFFu, got)) { ok = false; break; }
          grant_parity ^= 1u << stage;
          // This page's codes have landed; convert them key by key from the buffer. The loop is
          // kept rolled: four code regions share each scheduler's instruction cache, and the
          // unrolled conversion (~9 KB) made instruction fetch every role's top stall.
          ptx::cp_async_wait_all();
          __syncwarp();
          uint8_t* own_g = sm + kSmKv + stage * kStageBytes + cw * kOwnGroupBytes;
#pragma unroll 1
          for (int i = 0; i < 8; ++i) {
            const uint4 c = *reinterpret_cast<const uint4*>(raw_p + (lane >> 3) * kAtomBytes +
                                                            i * 128 + (lane & 7) * 16);
            const float sc = *reinterpret_cast<const float*>(rsc_p + i * 16 + (lane >> 3) * 4);
            uint4 lo, hi;
            lo.x = ptx::e4m3x2_scaled_bf16x2(c.x, sc);
            lo.y = ptx::e4m3x2_scaled_bf16x2(c.x >> 16, sc);
            lo.z = ptx::e4m3x2_scaled_bf16x2(c.y, sc);
            lo.w = ptx::e4m3x2_scaled_bf16x2(c.y >> 16, sc);
            hi.x = ptx::e4m3x2_scaled_bf16x2(c.z, sc);
            hi.y = ptx::e4m3x2_scaled_bf16x2(c.z >> 16, sc);
            hi.z = ptx::e4m3x2_scaled_bf16x2(c.w, sc);
            hi.w = ptx::e4m3x2_scaled_bf16x2(c.w >> 16, sc);
            // 16-byte units 2 (lane % 4) and + 1 of chunk lane / 4, row i, 128B-swizzled
            uint8_t* rowp = own_g + (lane >> 2) * kAtomBytes + i * 128;
            const int u0 = 2 * (lane & 3);
            *reinterpret_cast<uint4*>(rowp + ((u0 ^ i) << 4)) = lo;
            *reinterpret_cast<uint4*>(rowp + (((u0 + 1) ^ i) << 4)) = hi;
          }
          __syncwarp();  // the buffer is read: the next page's copies may overwrite it
          if (j + 1 < s.np) {
            issue(s.p0 + j + 1, nxt);
            if (j + 2 < s.np) fetch(s.p0 + j + 2, nxt);  // used one page from now
          }
          ptx::fence_proxy_async_smem();  // the MMAs and the bulk copy read through the async proxy
          __syncwarp();
          if (lane == 0) ptx::mbar_expect_tx(bar(kBarKvFull + stage), kPeerGroupBytes);
          wt.where = (8 << 24) | int(it & 0xFFFFFF);
          const bool free_peer =
              wt.wait<true>(bar(kBarPeerGrant + stage), (peer_parity >> stage) & 1u);
          if (!__all_sync(0xFFFFFFFFu, free_peer)) { ok = false; break; }
          peer_parity ^= 1u << stage;
          if (lane == 0) {
            const uint32_t src = base + kSmKv + stage * kStageBytes + cw * kOwnGroupBytes +
                                 peer_chunk0 * kAtomBytes;
            const uint32_t dst = ptx::map_peer(
                base + kSmKv + stage * kStageBytes + kPvxOffset + cw * kPeerGroupBytes, peer);
            ptx::bulk_copy_to_peer(dst, src, kPeerGroupBytes,
                                   ptx::map_peer(bar(kBarKvFull + stage), peer));
          }
          __syncwarp();
        }
      }
      ptx::cp_async_wait_all();  // no copy into this CTA stays in flight past this point
      __syncwarp();
    } else if constexpr (kSparse) {
      const int cw = warp - 6, hl = lane & 15;
      uint32_t it = 0;
      uint32_t grant_parity = 0;  // bit s: parity of the next grant phase of stage s
      // Sparse bf16: the next page's pool rows, read while this page's copies are in flight.
      int next_own[8], next_pr[4];
      bool have_next = false;
      int next_page = 0;  // dense: the segment's next page-table entry, read one page ahead
      Seg s;
      bool ok = true;
      while (ok && walker.next(meta, s)) {
        const int n = meta.unit_n[s.u];
        const int* pt = kSparse ? nullptr : a.page_table + (long long)a.seq_id[s.u] * a.slots;
        const int* srows = kSparse ? meta.sparse_rows + (long long)s.u * meta.topk : nullptr;
        it += 2;  // the segment's two query slots, filled by the TMA producer
        for (int j = 0; j < s.np; ++j, ++it) {
          const uint32_t stage = it % kStages;
          const int p = s.p0 + j;
          const int valid = min(kPageRows, n - p * kPageRows);
          long long row0 = 0;
          bool page_ok = true;
          if constexpr (!kSparse) {
            const int page = (have_next && j > 0) ? next_page : pt[p];
            if (j + 1 < s.np) next_page = pt[p + 1];  // used by the next page; no wait here
            have_next = j + 1 < s.np;
            row0 = (long long)page * kPageRows;
            page_ok = page >= 0 && row0 < a.pool_rows;
            if (!page_ok && cw == 0 && lane == 0)
              atomicOr(a.meta.header + kHdrError, TQ_DEV_PAGE_RANGE);
          }
          // Pool row of key k < valid of this page.
          auto row_of = [&](int k) -> long long {
            if constexpr (kSparse) return (long long)srows[p * kPageRows + k];
            else return row0 + k;
          };
          {
            // Sparse bf16 rows: the page's row numbers (read while the previous page of the
            // segment was in flight, else now), then the grant, then the copies.
            int own_row[8], pr_row[4];
            if (have_next) {
#pragma unroll
              for (int i = 0; i < 8; ++i) own_row[i] = next_own[i];
#pragma unroll
              for (int q = 0; q < 4; ++q) pr_row[q] = next_pr[q];
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int key = key0 + 8 * cw + i;
                own_row[i] = key < valid ? int(row_of(key)) : -1;
              }
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const int key = (kKeysPerCta - key0) + 8 * cw + 2 * q + (lane >> 4);
                pr_row[q] = key < valid ? int(row_of(key)) : -1;
              }
            }
            wt.where = (7 << 24) | int(it & 0xFFFFFF);
            const bool got =
                wt.wait<false>(bar(kBarKvGrant + stage), (grant_parity >> stage) & 1u);
            if (!__all_sync(0xFFFFFFFFu, got)) { ok = false; break; }
            grant_parity ^= 1u << stage;
            const uint32_t st_base = base + kSmKv + stage * kStageBytes;
            // Two 16-byte units (dims [8 u0, 8 u0 + 16) of the chunk) of one row; a row of -1
            // is written as zeros without a read.
            auto copy2 = [&](uint32_t rowp, int u0, int r8, int row, int byte0) {
              const uint8_t* src =
                  a.kv + (row < 0 ? 0 : (long long)row * a.kv_row_stride + byte0);
              const uint32_t nbytes = row < 0 ? 0u : 16u;
              ptx::cp_async_16(rowp + ((u0 ^ r8) << 4), src, nbytes);
              ptx::cp_async_16(rowp + (((u0 + 1) ^ r8) << 4), src + (row < 0 ? 0 : 16), nbytes);
            };
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int r = 8 * cw + i;
              copy2(st_base + (r >> 3) * kOwnGroupBytes + (lane >> 2) * kAtomBytes + (r & 7) * 128,
                    2 * (lane & 3), r & 7, own_row[i], 32 * lane);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int r = 8 * cw + 2 * q + (lane >> 4);
              copy2(st_base + kPvxOffset + (r >> 3) * kPeerGroupBytes + (hl >> 2) * kAtomBytes +
                        (r & 7) * 128,
                    2 * (hl & 3), r & 7, pr_row[q], 2 * vdim0 + 32 * hl);
            }
            have_next = j + 1 < s.np;
            if (have_next) {
              const int pn = p + 1;
              const int vn = min(kPageRows, n - pn * kPageRows);
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int key = key0 + 8 * cw + i;
                next_own[i] = key < vn ? srows[pn * kPageRows + key] : -1;
              }
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const int key = (kKeysPerCta - key0) + 8 * cw + 2 * q + (lane >> 4);
                next_pr[q] = key < vn ? srows[pn * kPageRows + key] : -1;
              }
            }
            ptx::cp_async_wait_all();
          }
          ptx::fence_proxy_async_smem();  // the MMAs read the stage through the async proxy
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(bar(kBarKvFull + stage));
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    // One thread per head row h (its TMEM lane), 32 own keys per page. Per page: scores to
    // log2 units, a candidate reference maximum (the running one, or the page maximum when that
    // grew by more than 2^8), probabilities against it, then one message to the peer: the bf16
    // probabilities and the candidate. The new running maximum is the larger of the running one
    // and both candidates; each CTA recomputes its own probabilities exactly against it and
    // rescales the peer's (only when a maximum moved). Both CTAs derive identical statistics.
    const int sw = warp - 2;                  // softmax warp index 0..3
    const int qd = warp & 3;                  // TMEM lane quarter
    const int h = 32 * qd + lane;
    const uint32_t lane_base = uint32_t(32 * qd) << 16;
    const uint32_t peer_base = ptx::map_peer(base + kSmPeer, peer);
    const uint32_t lsum_remote = ptx::map_peer(base + kSmLsum, peer) + 4u * h;
    const uint32_t msg_full_r = ptx::map_peer(bar(kBarMsgFull), peer);
    const uint32_t lsum_full_r = ptx::map_peer(bar(kBarLsumFull), peer);
    const float c2 = a.scale_log2;
    uint32_t it = 0, useq = 0;
    Seg s;
    bool ok = true;
    while (ok && walker.next(meta, s)) {
      const int n = meta.unit_n[s.u];
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < s.np; ++j) {
        const uint32_t itq = it + j, sb = itq & 1u, ph = (itq >> 1) & 1u;
        const int own_valid = min(kPageRows, n - (s.p0 + j) * kPageRows) - key0;
        wt.where = (3 << 24) | int(itq & 0xFFFFFF);
        if (!wt.wait<false>(bar(kBarSFull + sb), ph)) { ok = false; break; }
        __syncwarp();
        ptx::tc_fence_after();
        float sv[32];
        {
          uint32_t sr[32];
          const uint32_t t = tmem + lane_base + kTmemS + sb * 32;
          ptx::tmem_ld16(t, *reinterpret_cast<uint32_t(*)[16]>(&sr[0]));
          ptx::tmem_ld16(t + 16, *reinterpret_cast<uint32_t(*)[16]>(&sr[16]));
          ptx::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[i] = i < own_valid ? __uint_as_float(sr[i]) * c2 : -INFINITY;
        }
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < 32; ++i) mx = fmaxf(mx, sv[i]);
        const float m_cand = j == 0 ? mx : (mx > m_used + kRescaleThreshold ? mx : m_used);
        uint32_t pk[16];
        float l_page = 0.f;
        {
          float s0 = 0.f, s1 = 0.f;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float p0 = m_cand == -INFINITY ? 0.f : ptx::ex2(sv[2 * i] - m_cand);
            const float p1 = m_cand == -INFINITY ? 0.f : ptx::ex2(sv[2 * i + 1] - m_cand);
            pk[i] = ptx::pack_bf16x2(p0, p1);
            s0 += p0;
            s1 += p1;
          }
          l_page = s0 + s1;
        }
        // Send this page's probabilities and candidate once the peer's PV of page itq-2 has
        // consumed our previous message in that buffer (its MMA warp's commit arrives here).
        if (!wt.wait<true>(bar(kBarMsgFree + sb), ph ^ 1u)) { ok = false; break; }
        {
          const uint32_t dst = peer_base + sb * kPMsgBytes + 16u * h;
          const uint32_t rbar = msg_full_r + 8u * (sb * 4 + sw);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            ptx::st_async_v4(dst + c * kPChunkBytes, pk[4 * c], pk[4 * c + 1], pk[4 * c + 2],
                             pk[4 * c + 3], rbar);
          ptx::st_async_b32(peer_base + sb * kPMsgBytes + kPBytes + 4u * h,
                            __float_as_uint(m_cand), rbar);
        }
        if (!wt.wait<true>(bar(kBarMsgFull + sb * 4 + sw), ph)) { ok = false; break; }
        if (lane == 0) ptx::mbar_expect_tx(bar(kBarMsgFull + sb * 4 + sw), kWarpMsgBytes);
        const uint8_t* msg = sm + kSmPeer + sb * kPMsgBytes;
        const float m_peer = *reinterpret_cast<const float*>(msg + kPBytes + 4 * h);
        const float m_new = fmaxf(m_used, fmaxf(m_cand, m_peer));
        if (m_new != m_cand && m_cand != -INFINITY) {
          // Own probabilities against the new maximum, exactly (rare after the first page).
          float s0 = 0.f, s1 = 0.f;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float p0 = ptx::ex2(sv[2 * i] - m_new), p1 = ptx::ex2(sv[2 * i + 1] - m_new);
            pk[i] = ptx::pack_bf16x2(p0, p1);
            s0 += p0;
            s1 += p1;
          }
          l_page = s0 + s1;
        }
        if (m_new != m_peer && m_peer != -INFINITY) {
          // The peer's probabilities were against a smaller maximum: rescale them in place.
          const float f = ptx::ex2(m_peer - m_new);
          uint8_t* prow = sm + kSmPeer + sb * kPMsgBytes + 16 * h;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint4 v = *reinterpret_cast<uint4*>(prow + c * kPChunkBytes);
            v.x = ptx::pack_bf16x2(ptx::bf16_lo(v.x) * f, ptx::bf16_hi(v.x) * f);
            v.y = ptx::pack_bf16x2(ptx::bf16_lo(v.y) * f, ptx::bf16_hi(v.y) * f);
            v.z = ptx::pack_bf16x2(ptx::bf16_lo(v.z) * f, ptx::bf16_hi(v.z) * f);
            v.w = ptx::pack_bf16x2(ptx::bf16_lo(v.w) * f, ptx::bf16_hi(v.w) * f);
            *reinterpret_cast<uint4*>(prow + c * kPChunkBytes) = v;
          }
        }
        ptx::fence_proxy_async_smem();  // the peer's P (as received or rescaled) feeds the MMA
        float corr = 1.f;
        if (j > 0 && m_new > m_used) corr = ptx::ex2(m_used - m_new);
        l = l * corr + l_page;
        m_used = m_new;
        // The running maximum moved for some row of this warp: rescale those rows of O once
        // PV(itq-1) has landed. The decision is per lane but tcgen05.ld/st are warp-collective,
        // so the whole warp takes the branch (a factor of exactly 1 leaves a row unchanged).
        if (__any_sync(0xFFFFFFFFu, corr != 1.f)) {
          const uint32_t prev = itq - 1;
          if (!wt.wait<false>(bar(kBarPvDone + (prev & 1u)), (prev >> 1) & 1u)) { ok = false; break; }
          __syncwarp();
          ptx::tc_fence_after();
          for (int c = 0; c < kValueHalf; c += 16) {
            uint32_t v[16];
            ptx::tmem_ld16(tmem + lane_base + kTmemO + c, v);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * corr);
            ptx::tmem_st16(tmem + lane_base + kTmemO + c, v);
          }
          ptx::tmem_wait_st();
        }
        // Own P over the scores of this buffer (this thread read them above).
        __syncwarp();
        ptx::tmem_st16(tmem + lane_base + kTmemS + sb * 32, pk);
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(bar(kBarPFull + sb));
      }
      if (!ok) break;
      // Epilogue: the row sum over both CTAs' keys, then this CTA's 256 columns of O.
      wt.where = (5 << 24) | int(useq & 0xFFFFFF);
      ptx::st_async_b32(lsum_remote, __float_as_uint(l), lsum_full_r + 8u * sw);
      if (!wt.wait<true>(bar(kBarLsumFull + sw), useq & 1u)) break;
      const float l_peer = *reinterpret_cast<const float*>(sm + kSmLsum + 4 * h);
      __syncwarp();
      if (lane == 0) ptx::mbar_expect_tx(bar(kBarLsumFull + sw), 32 * 4);
      const float l_tot = rank == 0 ? l + l_peer : l_peer + l;
      if (!wt.wait<false>(bar(kBarOFull), useq & 1u)) break;
      __syncwarp();
      ptx::tc_fence_after();
      const float inv_l = 1.f / l_tot;
      if (rank == 0 && h < a.heads) {
        const float lse = (m_used + log2f(l_tot)) * kLn2;
        if (s.slot >= 0) meta.part_lse[(long long)s.slot * kHeadsTile + h] = lse;
        else a.lse[(long long)s.u * a.heads + h] = lse;
      }
      // O leaves TMEM 32 columns at a time, the next chunk's load in flight while this one is
      // stored. Split partials use the layout [slot][column quad][row] (float4), so each warp
      // store writes 32 consecutive rows' quads: 512 contiguous bytes.
      uint32_t v[2][32];
      __syncwarp();
      ptx::tmem_ld16(tmem + lane_base + kTmemO, *reinterpret_cast<uint32_t(*)[16]>(&v[0][0]));
      ptx::tmem_ld16(tmem + lane_base + kTmemO + 16, *reinterpret_cast<uint32_t(*)[16]>(&v[0][16]));
      ptx::tmem_wait_ld();
#pragma unroll
      for (int ci = 0; ci < kValueHalf / 32; ++ci) {
        const int c = 32 * ci;
        const uint32_t(&cur)[32] = v[ci & 1];
        if (ci + 1 < kValueHalf / 32) {
          __syncwarp();  // TMEM loads are warp-collective; lanes past the head count rejoin here
          ptx::tmem_ld16(tmem + lane_base + kTmemO + c + 32,
                         *reinterpret_cast<uint32_t(*)[16]>(&v[(ci + 1) & 1][0]));
          ptx::tmem_ld16(tmem + lane_base + kTmemO + c + 48,
                         *reinterpret_cast<uint32_t(*)[16]>(&v[(ci + 1) & 1][16]));
        }
        if (h >= a.heads) {
          // padding row: nothing to store
        } else if (s.slot >= 0) {
          float4* dst = reinterpret_cast<float4*>(meta.part_out) +
                        ((long long)s.slot * (kValueDim / 4) + (vdim0 + c) / 4) * kHeadsTile + h;
#pragma unroll
          for (int k = 0; k < 8; ++k)
            dst[k * kHeadsTile] = make_float4(__uint_as_float(cur[4 * k]) * inv_l,
                                              __uint_as_float(cur[4 * k + 1]) * inv_l,
                                              __uint_as_float(cur[4 * k + 2]) * inv_l,
                                              __uint_as_float(cur[4 * k + 3]) * inv_l);
        } else if (a.out_f32) {
          float4* dst = reinterpret_cast<float4*>(a.out + s.u * a.out_stride_t +
                                                  h * a.out_stride_h + (long long)(vdim0 + c) * 4);
#pragma unroll
          for (int k = 0; k < 8; ++k)
            dst[k] = make_float4(__uint_as_float(cur[4 * k]) * inv_l,
                                 __uint_as_float(cur[4 * k + 1]) * inv_l,
                                 __uint_as_float(cur[4 * k + 2]) * inv_l,
                                 __uint_as_float(cur[4 * k + 3]) * inv_l);
        } else {
          uint32_t pkd[16];
#pragma unroll
          for (int k = 0; k < 16; ++k)
            pkd[k] = ptx::pack_bf16x2(__uint_as_float(cur[2 * k]) * inv_l,
                                      __uint_as_float(cur[2 * k + 1]) * inv_l);
          uint4* dst = reinterpret_cast<uint4*>(a.out + s.u * a.out_stride_t +
                                                h * a.out_stride_h + (long long)(vdim0 + c) * 2);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            dst[k] = make_uint4(pkd[4 * k], pkd[4 * k + 1], pkd[4 * k + 2], pkd[4 * k + 3]);
        }
        if (ci + 1 < kValueHalf / 32) ptx::tmem_wait_ld();
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar(kBarOFree));
      it += s.np;
      ++useq;
    }
    // The peer's last releases of our message buffers arrive asynchronously (when its last PVs
    // complete); both have landed before this CTA may exit.
    for (uint32_t b = 0; b < 2 && b < it; ++b) {
      const uint32_t uses = (it + 1 - b) / 2;
      wt.wait<true>(bar(kBarMsgFree + b), (uses - 1) & 1u);
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  // Every message, row sum and buffer release between the pair has been awaited by its receiver,
  // so the exit barrier need not wait for this CTA's output stores to drain. After a timeout a
  // remote abort flag may still be in flight: then the full barrier orders it first.
  if (*abort_flag) {
    // After a timeout, copies and remote stores may still be in flight towards this CTA's
    // shared memory: give them a bounded 20 ms to land before the CTA leaves.
    const uint64_t t0 = ptx::global_timer_ns();
    for (uint32_t i = 0; i < (1u << 16) && ptx::global_timer_ns() - t0 < 20000000ull; ++i)
      __nanosleep(1000);
    ptx::cluster_sync();
  } else {
    ptx::cluster_sync_relaxed();
  }
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------
// Combine of split tokens, and zero-fill of tokens with no visible key.

__device__ __forceinline__ void store8(char* base, int f32, const float (&v)[8]) {
  if (f32) {
    float4* d = reinterpret_cast<float4*>(base);
    d[0] = make_float4(v[0], v[1], v[2], v[3]);
    d[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    *reinterpret_cast<uint4*>(base) =
        make_uint4(ptx::pack_bf16x2(v[0], v[1]), ptx::pack_bf16x2(v[2], v[3]),
                   ptx::pack_bf16x2(v[4], v[5]), ptx::pack_bf16x2(v[6], v[7]));
  }
}

// One thread per (split token, head, 8 value dims), grid-stride over a fixed grid. Each thread
// merges its 8 dims over the token's partials four at a time: the loads of four partials are in
// flight together, folded into a running maximum and sum of weights. Tokens that see no key are
// zero-filled by the same grid.
constexpr int kCombineBlocksPerPair = 16;

__global__ void __launch_bounds__(256) combine_kernel(Meta m, char* out, long long st_t,
                                                      long long st_h, int out_f32, float* lse,
                                                      int heads) {
  ptx::grid_dependency_wait();  // launched early; the attention kernel's results start here
  const int ncomb = m.header[kHdrNumCombine], nempty = m.header[kHdrNumEmpty];
  const int esize = out_f32 ? 4 : 2;
  const long long items = (long long)ncomb * heads * 64;
  for (long long t = blockIdx.x * 256ll + threadIdx.x; t < items; t += (long long)gridDim.x * 256) {
    // Consecutive threads take consecutive rows of one 8-column group: the partials'
    // [slot][column quad][row] layout makes their loads contiguous.
    const int job = int(t / (heads * 64)), rem = int(t % (heads * 64));
    const int h = rem % heads, d0 = (rem / heads) * 8;
    const int u = m.combine_list[job];
    const int ns = m.unit_nsplit[u], off = m.unit_split_off[u];
    float mx = -INFINITY, wsum = 0.f;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i0 = 0; i0 < ns; i0 += 4) {
      float li[4];
      float4 x[4][2];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (i0 + k < ns) {
          const long long slot = off + i0 + k;
          li[k] = __ldcg(m.part_lse + slot * kHeadsTile + h);
          const float4* src = reinterpret_cast<const float4*>(m.part_out) +
                              (slot * (kValueDim / 4) + d0 / 4) * kHeadsTile + h;
          x[k][0] = __ldcg(src);
          x[k][1] = __ldcg(src + kHeadsTile);
        } else {
          li[k] = -INFINITY;
          x[k][0] = x[k][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      const float m4 = fmaxf(fmaxf(li[0], li[1]), fmaxf(li[2], li[3]));
      if (m4 > mx) {
        const float f = mx == -INFINITY ? 0.f : expf(mx - m4);
        wsum *= f;
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] *= f;
        mx = m4;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float w = li[k] == -INFINITY ? 0.f : expf(li[k] - mx);
        wsum += w;
        acc[0] += w * x[k][0].x; acc[1] += w * x[k][0].y;
        acc[2] += w * x[k][0].z; acc[3] += w * x[k][0].w;
        acc[4] += w * x[k][1].x; acc[5] += w * x[k][1].y;
        acc[6] += w * x[k][1].z; acc[7] += w * x[k][1].w;
      }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] *= inv;
    store8(out + u * st_t + h * st_h + (long long)d0 * esize, out_f32, acc);
    // -inf only for an empty weight sum: a NaN partial (a NaN in a visible row) stays NaN.
    if (d0 == 0) lse[(long long)u * heads + h] = wsum == 0.f ? -INFINITY : mx + logf(wsum);
  }
  // Tokens with no visible key: zeros and lse = -inf.
  const float z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const long long tasks = (long long)nempty * heads * 64;
  for (long long t = blockIdx.x * 256ll + threadIdx.x; t < tasks; t += (long long)gridDim.x * 256) {
    const int e = int(t / (heads * 64));
    const int rem = int(t % (heads * 64));
    const int u = m.empty_list[e], h = rem >> 6, d0 = (rem & 63) * 8;
    store8(out + u * st_t + h * st_h + (long long)d0 * esize, out_f32, z);
    if (d0 == 0) lse[(long long)u * heads + h] = -INFINITY;
  }
}

// Merge of G per-device partial results (cross-device split of one sequence's pages).
__global__ void __launch_bounds__(256) merge_parts_kernel(const float* __restrict__ part_out,
                                                          const float* __restrict__ part_lse,
                                                          long long parts, long long tokens,
                                                          long long heads, char* out,
                                                          long long st_t, long long st_h,
                                                          int out_f32, float* lse) {
  const long long rows = tokens * heads;
  const int esize = out_f32 ? 4 : 2;
  for (long long task = blockIdx.x * (long long)blockDim.x + threadIdx.x; task < rows * 64;
       task += (long long)gridDim.x * blockDim.x) {
    const long long row = task >> 6;
    const int d0 = int(task & 63) * 8;
    const long long t = row / heads, h = row % heads;
    float mx = -INFINITY;
    for (long long g = 0; g < parts; ++g) mx = fmaxf(mx, part_lse[g * rows + row]);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float wsum = 0.f;
    for (long long g = 0; g < parts; ++g) {
      const float li = part_lse[g * rows + row];
      const float w = li == -INFINITY ? 0.f : expf(li - mx);
      if (w == 0.f) continue;
      wsum += w;
      const float4* src = reinterpret_cast<const float4*>(part_out + (g * rows + row) * kValueDim + d0);
      const float4 x0 = src[0], x1 = src[1];
      acc[0] += w * x0.x; acc[1] += w * x0.y; acc[2] += w * x0.z; acc[3] += w * x0.w;
      acc[4] += w * x1.x; acc[5] += w * x1.y; acc[6] += w * x1.z; acc[7] += w * x1.w;
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] *= inv;
    store8(out + t * st_t + h * st_h + (long long)d0 * esize, out_f32, acc);
    if (d0 == 0) lse[row] = wsum == 0.f ? -INFINITY : mx + logf(wsum);  // NaN stays NaN
  }
}

// ---------------------------------------------------------------------------------------------
// Seeded synthetic inputs (device). Same stream and transform as the host generator.

__device__ __forceinline__ void philox_block_dev(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3,
                                                 uint32_t k0, uint32_t k1, uint32_t (&o)[4]) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
    const uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c1 = lo1;
    c3 = lo0;
    c0 = n0;
    c2 = n2;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  o[0] = c0; o[1] = c1; o[2] = c2; o[3] = c3;
}

// Round a finite double to bf16 bits, nearest with ties to even, straight from its bit pattern.
__device__ __forceinline__ uint16_t double_to_bf16_bits(double x) {
  unsigned long long b = __double_as_longlong(x);
  const unsigned long long lsb = (b >> 45) & 1ull;
  b += ((1ull << 44) - 1ull) + lsb;
  b = (b >> 45) << 45;
  const float f = float(__longlong_as_double(b));  // exact: at most 8 significant bits
  return uint16_t(__float_as_uint(f) >> 16);
}

// Normal number `idx` of a stream: Box-Muller on words 2 idx and 2 idx + 1.
__device__ __forceinline__ uint16_t normal_bf16_dev(uint64_t seed, uint64_t stream, uint64_t idx) {
  const uint64_t w = 2 * idx, group = w >> 2;
  uint32_t o[4];
  philox_block_dev(uint32_t(group), uint32_t(group >> 32), uint32_t(stream), uint32_t(stream >> 32),
                   uint32_t(seed), uint32_t(seed >> 32), o);
  const uint32_t w0 = (w & 2) ? o[2] : o[0], w1 = (w & 2) ? o[3] : o[1];
  const double u1 = (double(w0 >> 8) + 1.0) * (1.0 / 16777216.0);
  const double u2 = double(w1 >> 8) * (1.0 / 16777216.0);
  const double z = sqrt(-2.0 * log(u1)) * cos(2.0 * 3.141592653589793 * u2);
  return double_to_bf16_bits(z);
}

__global__ void gen_normal_kernel(uint16_t* dst, uint64_t count, uint64_t seed, uint64_t stream,
                                  uint64_t start) {
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < count;
       i += uint64_t(gridDim.x) * blockDim.x)
    dst[i] = normal_bf16_dev(seed, stream, start + i);
}

__global__ void fill_u16_kernel(uint16_t* dst, uint64_t count, uint16_t v) {
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < count;
       i += uint64_t(gridDim.x) * blockDim.x)
    dst[i] = v;
}

// grid (sequences, 64): block (b, y) writes positions y, y + 64, ... of sequence b.
__global__ void gen_kv_rows_kernel(char* pool, uint64_t row_stride, uint64_t width,
                                   const int* __restrict__ page_table, uint64_t slots,
                                   const int* __restrict__ kv_len,
                                   const long long* __restrict__ tok_off, uint64_t seed,
                                   uint64_t stream, uint64_t pool_pages) {
  const int b = blockIdx.x;
  const long long n = kv_len[b];
  for (long long p = blockIdx.y; p < n; p += gridDim.y) {
    const int page = page_table[(long long)b * slots + p / kPageRows];
    if (page < 0 || uint64_t(page) >= pool_pages) continue;
    uint16_t* row = reinterpret_cast<uint16_t*>(
        pool + (uint64_t(page) * kPageRows + uint64_t(p % kPageRows)) * row_stride);
    const uint64_t e0 = (uint64_t(tok_off[b]) + uint64_t(p)) * width;
    for (uint64_t d = threadIdx.x; d < width; d += blockDim.x)
      row[d] = normal_bf16_dev(seed, stream, e0 + d);
  }
}

// ---------------------------------------------------------------------------------------------
// Host glue.

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool encode_bf16(CUtensorMap* map, const void* addr, int rank, const cuuint64_t* dims,
                 const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, cuuint32_t(rank), const_cast<void*>(addr), dims,
            strides, box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool kRope, bool kFp8 = false, bool kSparse = false>
cudaError_t prepare_kernel() {
  return cudaFuncSetAttribute(mla_paged_kernel<kRope, kFp8, kSparse>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmBytes));
}

// CTA pairs that are co-resident on `device` (the persistent grid size).
int pairs_for_device(int device) {
  static std::mutex mu;
  static int cache[128] = {0};
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0 || device >= 128) return 0;
  if (cache[device]) return cache[device];
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return 0;
  if (prev != device && cudaSetDevice(device) != cudaSuccess) return 0;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  int clusters = 0;
  if (prepare_kernel<true>() == cudaSuccess && prepare_kernel<false>() == cudaSuccess &&
      prepare_kernel<false, true>() == cudaSuccess &&
      prepare_kernel<false, false, true>() == cudaSuccess &&
      prepare_kernel<false, true, true>() == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&clusters, mla_paged_kernel<true>, &cfg) != cudaSuccess)
      clusters = 0;
  }
  cudaGetLastError();
  if (prev != device) cudaSetDevice(prev);
  if (clusters <= 0) return 0;
  cache[device] = clusters;
  return clusters;
}

uint64_t align256(uint64_t x) { return (x + 255) & ~uint64_t(255); }

void layout_for(uint64_t tokens, int pairs, bool sparse, uint64_t topk, TqWorkspaceLayout* L) {
  uint64_t o = 0;
  auto take = [&](uint64_t bytes) {
    const uint64_t at = o;
    o = align256(o + bytes);
    return at;
  };
  std::memset(L, 0, sizeof(*L));
  L->header = take(kHdrWords * 4);
  L->unit_n = take(tokens * 4);
  L->unit_pages = take(tokens * 4);
  L->unit_gstart = take(tokens * 4);
  L->unit_first = take(tokens * 4);
  L->unit_nsplit = take(tokens * 4);
  L->unit_split_off = take(tokens * 4);
  L->pair_begin = take(uint64_t(pairs) * 4);
  L->combine_list = take(tokens * 4);
  L->empty_list = take(tokens * 4);
  L->part_lse = take(uint64_t(2 * pairs) * kHeadsTile * 4);
  L->part_out = take(uint64_t(2 * pairs) * kHeadsTile * kValueDim * 4);
  if (sparse) {  // offsets never 0 (the header comes first), so 0 means "dense plan"
    L->sparse_rows = take(tokens * topk * 4);
    L->sparse_count = take(tokens * 4);
  }
  L->total_bytes = o;
  L->pairs = pairs;
}

Meta meta_at(char* ws, const TqWorkspaceLayout& L) {
  Meta m;
  m.header = reinterpret_cast<int*>(ws + L.header);
  m.unit_n = reinterpret_cast<int*>(ws + L.unit_n);
  m.unit_pages = reinterpret_cast<int*>(ws + L.unit_pages);
  m.unit_gstart = reinterpret_cast<int*>(ws + L.unit_gstart);
  m.unit_first = reinterpret_cast<int*>(ws + L.unit_first);
  m.unit_nsplit = reinterpret_cast<int*>(ws + L.unit_nsplit);
  m.unit_split_off = reinterpret_cast<int*>(ws + L.unit_split_off);
  m.pair_begin = reinterpret_cast<int*>(ws + L.pair_begin);
  m.combine_list = reinterpret_cast<int*>(ws + L.combine_list);
  m.empty_list = reinterpret_cast<int*>(ws + L.empty_list);
  m.part_lse = reinterpret_cast<float*>(ws + L.part_lse);
  m.part_out = reinterpret_cast<float*>(ws + L.part_out);
  m.sparse_rows = L.sparse_rows ? reinterpret_cast<int*>(ws + L.sparse_rows) : nullptr;
  m.sparse_count = L.sparse_count ? reinterpret_cast<int*>(ws + L.sparse_count) : nullptr;
  m.topk = 0;
  return m;
}

int32_t set_err(TqContractError* err, const char* field, int32_t kind) {
  if (err) {
    err->field = field;
    err->kind = kind;
  }
  return kind;
}

// Optional events recorded on the launch stream right before and right after the attention
// kernel (per calling thread; both null = off). Instrumentation for measuring the kernel alone.
thread_local cudaEvent_t t_timer_begin = nullptr;
thread_local cudaEvent_t t_timer_end = nullptr;

int32_t launch(const TqMlaParams* params, void* workspace, uint64_t workspace_bytes, void* stream,
               TqContractError* err) {
  if (!params_intact(params)) return set_err(err, "params", TQ_ERR_PARAMS);
  set_err(err, nullptr, TQ_OK);
  if (!params->should_launch) return TQ_OK;
  const TqMlaSpec& s = params->spec;
  const bool rope = s.kv_format == TQ_KV_BF16_ROPE576;
  const bool fp8 = s.kv_format == TQ_KV_FP8_E4M3;
  const bool sparse = params->sparse != 0;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return set_err(err, "device", TQ_ERR_CUDA);
  const int pairs = pairs_for_device(device);
  if (pairs <= 0) return set_err(err, "device", TQ_ERR_CUDA);
  TqWorkspaceLayout L;
  layout_for(params->tokens, pairs, params->sparse != 0, params->topk, &L);
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255) ||
      workspace_bytes < L.total_bytes)
    return set_err(err, "workspace", TQ_ERR_WORKSPACE);
  // TMA needs 16-byte aligned addresses and strides for q (natural alignment is 2 bytes).
  if (s.q.device_address % 16) return set_err(err, "q", TQ_ALIGNMENT);
  if (s.q.strides_bytes[0] % 16 || s.q.strides_bytes[1] % 16) return set_err(err, "q", TQ_STRIDE);
  const uint64_t pool_rows = params->pages * kPageRows;
  if (pool_rows >= (uint64_t(1) << 31) - kPageRows || params->tokens >= (uint64_t(1) << 31))
    return set_err(err, "kv", TQ_ERR_UNSUPPORTED);
  if (s.out.dtype == TQ_DTYPE_BF16 && (s.out.device_address % 16 || s.out.strides_bytes[0] % 16 ||
                                       s.out.strides_bytes[1] % 16))
    return set_err(err, "out", TQ_ALIGNMENT);
  if (s.out.dtype == TQ_DTYPE_F32 && (s.out.device_address % 16 || s.out.strides_bytes[0] % 16 ||
                                      s.out.strides_bytes[1] % 16))
    return set_err(err, "out", TQ_ALIGNMENT);

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  Meta m = meta_at(ws, L);
  const int T = int(params->tokens), H = int(params->heads), S = int(params->sequences);
  if (sparse) {
    m.topk = (long long)params->topk;
    const int blocks = T < 8 * pairs ? T : 8 * pairs;
    sparse_compact_kernel<<<blocks, 256, 0, st>>>(
        m, reinterpret_cast<const int*>(params->idx.device_address),
        (long long)(params->idx.strides_bytes[0] / 4),
        reinterpret_cast<const int*>(params->k_len.device_address),
        reinterpret_cast<const int*>(s.seq_id.device_address),
        reinterpret_cast<const int*>(s.q_pos.device_address),
        reinterpret_cast<const int*>(s.kv_len.device_address),
        reinterpret_cast<const int*>(s.page_table.device_address), (long long)params->slots,
        (long long)params->pages, S, T);
  }

  schedule_kernel<<<1, 1024, 0, st>>>(m, reinterpret_cast<const int*>(s.seq_id.device_address),
                                      reinterpret_cast<const int*>(s.q_pos.device_address),
                                      reinterpret_cast<const int*>(s.kv_len.device_address), T,
                                      S, (long long)params->slots, (long long)params->pages,
                                      pairs);
  if (params->pages > 0) {
    CUtensorMap tq_map, tkv, tv;
    const uint64_t width = params->qk_width;
    const cuuint64_t qdims[3] = {width, params->heads, params->tokens};
    const cuuint64_t qstr[2] = {s.q.strides_bytes[1], s.q.strides_bytes[0]};
    const cuuint32_t qbox[3] = {64, cuuint32_t(kHeadsTile), 1};
    // Pool rows seen as {64 dims, row in an 8-row group, 64-dim chunk, 8-row group}: strides
    // row_stride, 128 B and 8 rows. A box reads whole 8-row groups (contiguous bytes) at a time
    // and lands as [group][chunk][8 rows x 128 B], a 128B-swizzled UMMA operand layout.
    const cuuint64_t kdims[4] = {64, 8, width / 64, pool_rows / 8};
    const cuuint64_t kstr[3] = {params->row_stride, 128, 8 * params->row_stride};
    const cuuint32_t kbox[4] = {64, 8, uint32_t(width / 64), uint32_t(kKeysPerCta / 8)};
    const cuuint32_t vbox[4] = {64, 8, uint32_t(kValueHalf / 64), uint32_t(kKeysPerCta / 8)};
    const void* qa = reinterpret_cast<const void*>(s.q.device_address);
    const void* ka = reinterpret_cast<const void*>(s.kv.device_address);
    if (!encode_bf16(&tq_map, qa, 3, qdims, qstr, qbox, CU_TENSOR_MAP_SWIZZLE_128B))
      return set_err(err, "tensor_map", TQ_ERR_CUDA);
    if (fp8 || sparse) {
      tkv = tq_map;  // the convert warps gather the rows: the KV maps are not used
      tv = tq_map;
    } else if (!encode_bf16(&tkv, ka, 4, kdims, kstr, kbox, CU_TENSOR_MAP_SWIZZLE_128B) ||
               !encode_bf16(&tv, ka, 4, kdims, kstr, vbox, CU_TENSOR_MAP_SWIZZLE_128B)) {
      return set_err(err, "tensor_map", TQ_ERR_CUDA);
    }
    MainArgs a;
    a.meta = m;
    a.q = reinterpret_cast<const char*>(s.q.device_address);
    a.q_stride_t = (long long)s.q.strides_bytes[0];
    a.q_stride_h = (long long)s.q.strides_bytes[1];
    a.page_table = reinterpret_cast<const int*>(s.page_table.device_address);
    a.seq_id = reinterpret_cast<const int*>(s.seq_id.device_address);
    a.slots = (long long)params->slots;
    a.pool_rows = (long long)pool_rows;
    a.tokens = T;
    a.heads = H;
    a.out = reinterpret_cast<char*>(s.out.device_address);
    a.out_stride_t = (long long)s.out.strides_bytes[0];
    a.out_stride_h = (long long)s.out.strides_bytes[1];
    a.out_f32 = s.out.dtype == TQ_DTYPE_F32;
    a.lse = reinterpret_cast<float*>(s.lse.device_address);
    a.scale_log2 = s.softmax_scale * 1.4426950408889634f;
    a.kv = reinterpret_cast<const uint8_t*>(s.kv.device_address);
    a.kv_row_stride = (long long)params->row_stride;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    cfg.blockDim = dim3((fp8 || sparse) ? kThreadsGather : kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (t_timer_begin && cudaEventRecord(t_timer_begin, st) != cudaSuccess)
      return set_err(err, "timer", TQ_ERR_CUDA);
    cudaError_t e;
    if (rope)
      e = cudaLaunchKernelEx(&cfg, mla_paged_kernel<true>, tq_map, tkv, tv, a);
    else if (sparse && fp8)
      e = cudaLaunchKernelEx(&cfg, mla_paged_kernel<false, true, true>, tq_map, tkv, tv, a);
    else if (sparse)
      e = cudaLaunchKernelEx(&cfg, mla_paged_kernel<false, false, true>, tq_map, tkv, tv, a);
    else if (fp8)
      e = cudaLaunchKernelEx(&cfg, mla_paged_kernel<false, true>, tq_map, tkv, tv, a);
    else
      e = cudaLaunchKernelEx(&cfg, mla_paged_kernel<false>, tq_map, tkv, tv, a);
    if (e != cudaSuccess) return set_err(err, "launch", TQ_ERR_CUDA);
    if (t_timer_end && cudaEventRecord(t_timer_end, st) != cudaSuccess)
      return set_err(err, "timer", TQ_ERR_CUDA);
  }
  {
    // Launched as a programmatic dependent of the attention kernel (or of the scheduler when
    // there is no page): its blocks start early and wait inside the kernel.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pairs * kCombineBlocksPerPair, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, combine_kernel, m, reinterpret_cast<char*>(s.out.device_address),
                           (long long)s.out.strides_bytes[0], (long long)s.out.strides_bytes[1],
                           int(s.out.dtype == TQ_DTYPE_F32),
                           reinterpret_cast<float*>(s.lse.device_address), H) != cudaSuccess)
      return set_err(err, "launch", TQ_ERR_CUDA);
  }
  if (cudaGetLastError() != cudaSuccess) return set_err(err, "launch", TQ_ERR_CUDA);
  return TQ_OK;
}

// ---------------------------------------------------------------------------------------------
// Fixed scratch for callers that cannot allocate device memory (see tq_mla_decode_no_alloc).
// Every GPU that loads this library holds these TQ_MLA_NO_ALLOC_WORKSPACE_BYTES until exit.

static __device__ __align__(256) uint8_t g_no_alloc_workspace[TQ_MLA_NO_ALLOC_WORKSPACE_BYTES];

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

// Device address of g_no_alloc_workspace on `device` in the current context, looked up with
// that device current (in host code the array's name is only a host-side stand-in). The
// address is cached per device together with the context it was found in, and found again when
// the current context differs (a device reset, or a driver-API context other than the primary
// one), so a cached address is never used in another context.
void* no_alloc_workspace(int device) {
  static std::mutex mu;
  static void* cache[128] = {nullptr};
  static CUcontext cache_ctx[128] = {nullptr};
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0 || device >= 128) return nullptr;
  CUcontext ctx = nullptr;
  CtxGetCurrentFn get = ctx_get_current_fn();
  if (!get || get(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  if (!cache[device] || !ctx || cache_ctx[device] != ctx) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_no_alloc_workspace) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    if (!ctx && get && get(&ctx) != CUDA_SUCCESS) ctx = nullptr;  // made current by the lookup
    cache[device] = ptr;
    cache_ctx[device] = ctx;
  }
  return cache[device];
}

}  // namespace mla
}  // namespace tq

using namespace tq::mla;

extern "C" {

int32_t tq_mla_workspace_layout(const TqMlaParams* params, int32_t device,
                                TqWorkspaceLayout* layout) {
  if (!layout) return TQ_ERR_INVALID_ARGUMENT;
  if (!tq::params_intact(params)) return TQ_ERR_PARAMS;
  const int pairs = pairs_for_device(device);
  if (pairs <= 0) return TQ_ERR_CUDA;
  layout_for(params->tokens, pairs, params->sparse != 0, params->topk, layout);
  return TQ_OK;
}

int32_t tq_mla_workspace_bytes(const TqMlaParams* params, int32_t device, uint64_t* bytes) {
  if (!bytes) return TQ_ERR_INVALID_ARGUMENT;
  TqWorkspaceLayout L;
  const int32_t st = tq_mla_workspace_layout(params, device, &L);
  if (st != TQ_OK) return st;
  *bytes = L.total_bytes;
  return TQ_OK;
}

int32_t tq_mla_decode(const TqMlaParams* params, void* workspace, uint64_t workspace_bytes,
                      void* stream, TqContractError* err) {
  if (params && tq::params_intact(params) && params->max_queries_per_sequence == 0)
    return set_err(err, "params", TQ_ERR_PARAMS);  // a prefill plan
  return launch(params, workspace, workspace_bytes, stream, err);
}

int32_t tq_mla_decode_no_alloc(const TqMlaParams* params, void* stream, TqContractError* err) {
  if (!params || !tq::params_intact(params)) return set_err(err, "params", TQ_ERR_PARAMS);
  if (params->max_queries_per_sequence == 0) return set_err(err, "params", TQ_ERR_PARAMS);
  if (!params->should_launch) return set_err(err, nullptr, TQ_OK);
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return set_err(err, "device", TQ_ERR_CUDA);
  const int pairs = pairs_for_device(device);
  if (pairs <= 0) return set_err(err, "device", TQ_ERR_CUDA);
  TqWorkspaceLayout L;
  layout_for(params->tokens, pairs, params->sparse != 0, params->topk, &L);
  if (L.total_bytes > TQ_MLA_NO_ALLOC_WORKSPACE_BYTES)
    return set_err(err, "no_alloc_workspace", TQ_ERR_WORKSPACE);
  void* ws = no_alloc_workspace(device);
  if (!ws) return set_err(err, "no_alloc_workspace", TQ_ERR_CUDA);
  // The scheduler kernel rewrites every workspace word the later kernels read, so the previous
  // call's contents need no clearing.
  return launch(params, ws, TQ_MLA_NO_ALLOC_WORKSPACE_BYTES, stream, err);
}

int32_t tq_mla_no_alloc_read_device_error(void* stream, int32_t* flags) {
  if (!flags) return TQ_ERR_INVALID_ARGUMENT;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return TQ_ERR_CUDA;
  void* ws = no_alloc_workspace(device);
  if (!ws) return TQ_ERR_CUDA;
  // The header sits at offset 0 of every workspace layout.
  return tq_mla_read_device_error(ws, stream, flags);
}

int32_t tq_mla_prefill(const TqMlaParams* params, void* workspace, uint64_t workspace_bytes,
                       void* stream, TqContractError* err) {
  return launch(params, workspace, workspace_bytes, stream, err);
}

int32_t tq_mla_combine(const TqCombineParams* p, void* stream) {
  if (!p || !p->part_out || !p->part_lse || !p->out || !p->lse) return TQ_ERR_INVALID_ARGUMENT;
  if (p->parts == 0 || p->tokens == 0 || p->heads == 0) return TQ_OK;
  if ((p->part_out | p->out | p->out_stride_token | p->out_stride_head) % 16)
    return TQ_ALIGNMENT;
  const long long tasks = (long long)(p->tokens * p->heads * 64);
  const int blocks = int(std::min<long long>((tasks + 255) / 256, 148 * 8));
  merge_parts_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float*>(p->part_out), reinterpret_cast<const float*>(p->part_lse),
      (long long)p->parts, (long long)p->tokens, (long long)p->heads,
      reinterpret_cast<char*>(p->out), (long long)p->out_stride_token,
      (long long)p->out_stride_head, p->out_dtype == TQ_DTYPE_F32,
      reinterpret_cast<float*>(p->lse));
  return cudaGetLastError() == cudaSuccess ? TQ_OK : TQ_ERR_CUDA;
}

int32_t tq_mla_set_kernel_timer(void* begin_event, void* end_event) {
  if ((begin_event == nullptr) != (end_event == nullptr)) return TQ_ERR_INVALID_ARGUMENT;
  t_timer_begin = static_cast<cudaEvent_t>(begin_event);
  t_timer_end = static_cast<cudaEvent_t>(end_event);
  return TQ_OK;
}

int32_t tq_mla_read_device_error(const void* workspace, void* stream, int32_t* flags) {
  if (!workspace || !flags) return TQ_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t v = 0;
  if (cudaMemcpyAsync(&v, workspace, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return TQ_ERR_CUDA;
  *flags = v;
  return TQ_OK;
}

int32_t tq_gen_normal_bf16(void* dst, uint64_t count, uint64_t seed, uint64_t stream_id,
                           uint64_t start, void* stream) {
  if (!dst && count) return TQ_ERR_INVALID_ARGUMENT;
  if (!count) return TQ_OK;
  const uint64_t blocks = std::min<uint64_t>((count + 255) / 256, 148 * 16);
  gen_normal_kernel<<<unsigned(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint16_t*>(dst), count, seed, stream_id, start);
  return cudaGetLastError() == cudaSuccess ? TQ_OK : TQ_ERR_CUDA;
}

int32_t tq_gen_kv_pool(void* pool, uint64_t pool_pages, uint64_t row_stride, uint64_t width,
                       const void* page_table, uint64_t slots, const void* kv_len,
                       const void* tok_off, uint64_t sequences, uint64_t seed, void* stream) {
  if (!pool || row_stride % 2 || width * 2 > row_stride) return TQ_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint64_t halves = pool_pages * kPageRows * row_stride / 2;
  if (halves) {
    const uint64_t blocks = std::min<uint64_t>((halves + 255) / 256, 148 * 16);
    fill_u16_kernel<<<unsigned(blocks), 256, 0, st>>>(static_cast<uint16_t*>(pool), halves,
                                                      uint16_t(0x7FC0));
  }
  if (sequences && pool_pages) {
    gen_kv_rows_kernel<<<dim3(unsigned(sequences), 64), 256, 0, st>>>(
        static_cast<char*>(pool), row_stride, width, static_cast<const int*>(page_table), slots,
        static_cast<const int*>(kv_len), static_cast<const long long*>(tok_off), seed, 2,
        pool_pages);
  }
  return cudaGetLastError() == cudaSuccess ? TQ_OK : TQ_ERR_CUDA;
}

const char* tq_mla_version(void) { return "tq_mla 0.1.0 sm_100a"; }

}  // extern "C"
