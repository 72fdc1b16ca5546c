// Weight-streaming projections of the MLA prologue for decode-sized batches (T <= 128 tokens):
// out[T, N] = bf16(x[T, K] . w[N, K]^T), bf16 in, f32 accumulate.
//
// At decode sizes these GEMMs stream their weights once (tens of MB) against a few hundred KB of
// activations, so the weights are the MMA's M operand and the tokens its N. The kernel is
// persistent: one CTA per SM, grouped in clusters of S CTAs. A cluster walks over 128-row weight
// tiles (tile = cluster, cluster + clusters, ...); CTA r of the cluster always takes the r-th
// of S ranges of K. Per CTA:
//   warp 0 (one lane)  streams 128 x 64 weight boxes and T_pad x 64 token boxes (128-byte
//                      swizzle) through a ring of stages, continuing across tiles;
//   warp 1 (one lane)  issues tcgen05.mma (M = 128, N = T_pad, K = 16) into one of two TMEM
//                      accumulators (tile j into accumulator j % 2);
//   warps 2-5          move the finished accumulator into one of two f32 partial tiles in
//                      shared memory ([T_pad][128], token-major), tell every CTA of the cluster
//                      it is there, and then add, for the token rows r, r + S, ... of the tile,
//                      the S partials of the cluster in split order through distributed shared
//                      memory, round to bf16 and store the row.
// So the loads of tile j + 1 overlap the epilogue and reduction of tile j, and only the bf16
// output reaches global memory; the sums do not depend on timing.
// Hand-offs between CTAs are mbarriers in each CTA's shared memory: red_full[b] (S arrivals: the
// partial tiles b of all S CTAs are written) and red_free[b] (S arrivals: every CTA has read
// this CTA's partial tile b). All waits are bounded (2 s and a poll count); a timeout sets
// TQ_DEV_WAIT_TIMEOUT in the caller's device flags and the CTA skips its remaining waits.

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "tq_contracts.h"
#include "tq_ptx.cuh"

namespace tq {
namespace proj {

constexpr int kThreads = 192;
constexpr int kMaxStages = 8;
constexpr int kChunk = 64;                         // K elements per TMA box (128 bytes of bf16)
constexpr uint32_t kWBoxBytes = 128 * kChunk * 2;  // 16 KB
constexpr int kMaxTokens = kProjMaxTokens;
// One CTA per SM: the 227 KB a CTA may hold.
constexpr uint32_t kSmemBudget = 227u * 1024u;
constexpr uint32_t kSmemExtra = 1024 + 256;  // alignment slack, barriers and the TMEM address
constexpr uint64_t kWaitNs = 2000000000ull;

__host__ __device__ constexpr uint32_t stage_bytes(int tpad) {
  return kWBoxBytes + uint32_t(tpad) * kChunk * 2;
}
__host__ __device__ constexpr uint32_t red_bytes(int tpad) { return uint32_t(tpad) * 128 * 4; }

struct Args {
  int n, k, t, tpad;  // out features, reduction, tokens, tokens padded to 16
  int chunks;         // K boxes of 64
  int stages;         // ring depth, 2 to kMaxStages
  int splits;         // CTAs per cluster (K ranges)
  int tiles;          // 128-row weight tiles
  uint16_t* out;      // bf16 [T, N]
  int* flags;         // device error flags, may be null
};

struct Wait {
  int* flags;
  bool failed = false;
  template <bool kCluster = false>
  __device__ bool on(uint32_t bar, uint32_t parity) {
    if (failed) return false;
    auto test = [&] {
      return kCluster ? ptx::mbar_test_cluster(bar, parity) : ptx::mbar_test(bar, parity);
    };
    if (test()) return true;
    const uint64_t t0 = ptx::global_timer_ns();
    for (uint32_t i = 1;; ++i) {
      if (test()) return true;
      if ((i & 255) == 0 && (ptx::global_timer_ns() - t0 > kWaitNs || i > (1u << 26))) {
        if (flags) atomicOr(flags, TQ_DEV_WAIT_TIMEOUT);
        failed = true;
        return false;
      }
    }
  }
};

__device__ __forceinline__ uint2 pack_bf16x4(float x, float y, float z, float w) {
  uint32_t lo, hi;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(y), "f"(x));
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(w), "f"(z));
  return make_uint2(lo, hi);
}

// The four epilogue warps' own barrier (named barrier 1).
__device__ __forceinline__ void epilogue_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ void fence_acq_rel_cluster() {
  asm volatile("fence.acq_rel.cluster;" ::: "memory");
}

// Grid: `clusters` x S CTAs in clusters of S along x, one per SM, 192 threads.
template <int S>
__global__ void __launch_bounds__(kThreads, 1)
    proj_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                const Args a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = ptx::smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* sm = smem_raw + (base - raw);
  const int ns = a.stages;
  const uint32_t sb = stage_bytes(a.tpad), rb = red_bytes(a.tpad);
  const uint32_t red0 = base + uint32_t(ns) * sb;  // the two partial tiles
  const uint32_t bars = red0 + 2 * rb;
  // full[ns], empty[ns], then acc_full[2], acc_empty[2], red_full[2], red_free[2]
  auto full = [&](int s) { return bars + 8u * uint32_t(s); };
  auto empty = [&](int s) { return bars + 8u * uint32_t(ns + s); };
  auto acc_full = [&](int b) { return bars + 8u * uint32_t(2 * ns + b); };
  auto acc_empty = [&](int b) { return bars + 8u * uint32_t(2 * ns + 2 + b); };
  auto red_full = [&](int b) { return bars + 8u * uint32_t(2 * ns + 4 + b); };
  auto red_free = [&](int b) { return bars + 8u * uint32_t(2 * ns + 6 + b); };
  uint32_t* tmem_holder =
      reinterpret_cast<uint32_t*>(sm + (bars - base) + 8 * (2 * kMaxStages + 8));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = int(ptx::cluster_rank());
  const int cid = int(blockIdx.x) / S, nclusters = int(gridDim.x) / S;
  const int c0 = int((long long)rank * a.chunks / S);
  const int c1 = int((long long)(rank + 1) * a.chunks / S);
  const bool work = c1 > c0;
  const int ntiles = cid < a.tiles ? (a.tiles - cid + nclusters - 1) / nclusters : 0;
  const uint32_t x_bytes = uint32_t(a.tpad) * kChunk * 2;
  const uint32_t cols = a.tpad <= 32 ? 32u : a.tpad <= 64 ? 64u : 128u;  // per accumulator
  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      ptx::mbar_init(full(s), 1);
      ptx::mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(acc_full(b), 1);
      ptx::mbar_init(acc_empty(b), 4);
      ptx::mbar_init(red_full(b), uint32_t(S));
      ptx::mbar_init(red_free(b), uint32_t(S));
    }
    ptx::fence_mbar_init_cluster();
    ptx::tma_prefetch_desc(&tm_w);
    ptx::tma_prefetch_desc(&tm_x);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_addr(tmem_holder), 2 * cols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  ptx::cluster_sync();  // every CTA's barriers exist before any arrival from a peer
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  Wait wt{a.flags};
  if (warp == 0) {
    if (lane == 0 && work) {
      // Producer: for each tile, weight box {64 K, 128 rows} at (c * 64, tile * 128) and token
      // box {64, T_pad} at (c * 64, 0), c over this CTA's K range; the ring runs on across tiles.
      int i = 0;
      bool ok = true;
      for (int j = 0; j < ntiles && ok; ++j) {
        const int tile = cid + j * nclusters;
        for (int c = c0; c < c1; ++c, ++i) {
          const int s = i % ns;
          if (i >= ns && !wt.on(empty(s), uint32_t((i / ns) - 1) & 1u)) {
            ok = false;
            break;
          }
          const uint32_t dst = base + uint32_t(s) * sb;
          ptx::mbar_expect_tx(full(s), kWBoxBytes + x_bytes);
          ptx::tma_load_2d(dst, &tm_w, full(s), c * kChunk, tile * 128);
          ptx::tma_load_2d(dst + kWBoxBytes, &tm_x, full(s), c * kChunk, 0);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (work) {
      // MMA issuer: K-major operands, 128-byte swizzle (rows 128 B apart, 8-row groups 1 KB
      // apart); a K = 16 step advances the start address by 32 bytes inside the swizzle atom.
      const uint32_t idesc = ptx::idesc_bf16(128, uint32_t(a.tpad), 0);
      int i = 0;
      bool ok = true;
      for (int j = 0; j < ntiles && ok; ++j) {
        const int b = j & 1;
        if (j >= 2) {
          ok = __all_sync(0xFFFFFFFFu, wt.on(acc_empty(b), uint32_t((j >> 1) - 1) & 1u));
          if (!ok) break;
        }
        ptx::tc_fence_after();
        const uint32_t acc = tmem + uint32_t(b) * cols;
        for (int c = c0; c < c1; ++c, ++i) {
          const int s = i % ns;
          ok = __all_sync(0xFFFFFFFFu, wt.on(full(s), uint32_t(i / ns) & 1u));
          if (!ok) break;
          ptx::tc_fence_after();
          const uint32_t st = base + uint32_t(s) * sb;
          const uint64_t ad = ptx::smem_desc(st, 16, 1024, 2);
          const uint64_t bd = ptx::smem_desc(st + kWBoxBytes, 16, 1024, 2);
#pragma unroll
          for (int kk = 0; kk < kChunk / 16; ++kk)
            ptx::mma_ss_warp(acc, ad + uint64_t((kk * 32) >> 4), bd + uint64_t((kk * 32) >> 4),
                             idesc, (c > c0 || kk > 0) ? 1u : 0u);
          ptx::mma_commit_warp(empty(s));  // the stage may be refilled
        }
        ptx::mma_commit_warp(acc_full(b));  // accumulator b holds tile j
      }
    }
    __syncwarp();
  } else {
    // Epilogue warps 2-5: warp w may read TMEM lanes 32 (w % 4) .. 32 (w % 4) + 31.
    const int ew = warp - 2, quad = warp & 3, c4 = lane * 4;
    for (int j = 0; j < ntiles; ++j) {
      const int tile = cid + j * nclusters, b = j & 1;
      const uint32_t ph = uint32_t(j >> 1) & 1u;
      const uint32_t red = red0 + uint32_t(b) * rb;
      float* redp = reinterpret_cast<float*>(sm + (red - base));
      // Partial tile b was last read by the cluster for tile j - 2.
      bool ok = j < 2 || wt.on<true>(red_free(b), ph ^ 1u);
      if (work) ok = wt.on(acc_full(b), ph) && ok;
      ok = __all_sync(0xFFFFFFFFu, ok);
      ptx::tc_fence_after();
      if (ok && work) {
        const uint32_t acc = tmem + uint32_t(b) * cols + (uint32_t(quad * 32) << 16);
        for (int jj = 0; jj < a.tpad; jj += 16) {
          uint32_t r[16];
          ptx::tmem_ld16(acc + uint32_t(jj), r);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 16; ++q)
            redp[(jj + q) * 128 + quad * 32 + lane] = __uint_as_float(r[q]);
        }
      } else {
        for (int jj = 0; jj < a.tpad; ++jj) redp[jj * 128 + quad * 32 + lane] = 0.f;
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(acc_empty(b));  // accumulator b may take tile j + 2
      // Publish partial tile b to the cluster: after the epilogue warps' barrier, lane r of the
      // first epilogue warp fences at cluster scope (covering every store that barrier ordered
      // before it) and arrives on CTA r's red_full[b]; the S arrivals go out in parallel.
      epilogue_sync();
      if (ew == 0 && lane < S) {
        fence_acq_rel_cluster();
        ptx::mbar_arrive_cluster_relaxed(ptx::map_peer(red_full(b), uint32_t(lane)));
      }
      ok = __all_sync(0xFFFFFFFFu, wt.on<true>(red_full(b), ph));
      if (ok) {
        // Token rows rank + S (ew + 4 i), G at a time: the S partials of four consecutive
        // outputs of G rows, all loaded before any is added, then added in split order.
        constexpr int G = 16 / S;
        const int n0 = tile * 128 + c4;
        const int first = rank + S * ew;
        const int rows = a.t > first ? (a.t - first + 4 * S - 1) / (4 * S) : 0;
        for (int i0 = 0; i0 < rows; i0 += G) {
          float4 v[G * S];
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const int t = first + 4 * S * (i0 + g);
            const uint32_t off = red + uint32_t(t * 128 + c4) * 4u;
#pragma unroll
            for (int r = 0; r < S; ++r)
              if (i0 + g < rows) v[g * S + r] = ptx::ld_cluster_f4(ptx::map_peer(off, uint32_t(r)));
          }
#pragma unroll
          for (int g = 0; g < G; ++g) {
            if (i0 + g >= rows) break;
            const int t = first + 4 * S * (i0 + g);
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int r = 0; r < S; ++r) {
              acc.x += v[g * S + r].x;
              acc.y += v[g * S + r].y;
              acc.z += v[g * S + r].z;
              acc.w += v[g * S + r].w;
            }
            if (n0 < a.n)  // N is a multiple of 4: the four outputs are all in range or all out
              *reinterpret_cast<uint2*>(a.out + (long long)t * a.n + n0) =
                  pack_bf16x4(acc.x, acc.y, acc.z, acc.w);
          }
        }
      }
      // Every thread's reads of the cluster's partial tiles b have returned (their values are
      // stored above): each CTA may overwrite its partial tile b.
      epilogue_sync();
      if (ew == 0 && lane < S)
        ptx::mbar_arrive_cluster_relaxed(ptx::map_peer(red_free(b), uint32_t(lane)));
    }
    // Leave only once no CTA of the cluster reads this CTA's partial tiles any more.
    for (int b = 0; b < 2; ++b) {
      if (ntiles > b) {
        const int last = b + ((ntiles - 1 - b) / 2) * 2;
        wt.on<true>(red_free(b), uint32_t(last >> 1) & 1u);
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 2 * cols);
  }
}

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

// A packed bf16 [rows, k] matrix as a 2D map with {64, box_rows} boxes and 128-byte swizzle;
// rows past `rows` and columns past `k` read as zeros.
bool encode_rows(CUtensorMap* map, const void* addr, uint64_t rows, uint64_t k, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {k, rows};
  const cuuint64_t strides[1] = {k * 2};
  const cuuint32_t box[2] = {uint32_t(kChunk), box_rows};
  const cuuint32_t elem[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(addr), dims, strides, box,
            elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Ring depth for a token tile: what is left of the budget after the two partial tiles.
int stages_for(int tpad) {
  const uint64_t room = uint64_t(kSmemBudget) - kSmemExtra - 2ull * red_bytes(tpad);
  const int s = int(room / stage_bytes(tpad));
  return s > kMaxStages ? kMaxStages : s;
}

uint32_t smem_for(int tpad) {
  return uint32_t(stages_for(tpad)) * stage_bytes(tpad) + 2 * red_bytes(tpad) + kSmemExtra;
}

typedef void (*KernelFn)(const CUtensorMap, const CUtensorMap, const Args);

KernelFn kernel_for(int splits) {
  switch (splits) {
    case 1: return proj_kernel<1>;
    case 2: return proj_kernel<2>;
    case 3: return proj_kernel<3>;
    case 4: return proj_kernel<4>;
    case 5: return proj_kernel<5>;
    case 6: return proj_kernel<6>;
    case 7: return proj_kernel<7>;
    case 8: return proj_kernel<8>;
    default: return nullptr;
  }
}

// Clusters of S CTAs that fit on the device at once with this kernel's shared memory (one CTA
// per SM), asked of the occupancy calculator once per (device, S, token tile).
int max_clusters(int device, int splits, int tpad) {
  static std::mutex mu;
  static int cache[16][kProjMaxSplits + 1][kMaxTokens / 16 + 1] = {};
  if (device < 0 || device >= 16 || splits < 1 || splits > kProjMaxSplits) return 0;
  std::lock_guard<std::mutex> lock(mu);
  int& slot = cache[device][splits][tpad / 16];
  if (slot) return slot;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(splits), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_for(tpad);
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = unsigned(splits);
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel_for(splits), &cfg) != cudaSuccess) n = 0;
  slot = n;
  return n;
}

}  // namespace proj

int proj_splits(int n, int k, int t, int sms) {
  // A cluster of S CTAs takes ceil(tiles / clusters) tiles of ceil(chunks / S) K boxes each,
  // with about sms / S clusters resident; a CTA's fill and last reduction cost about four
  // boxes' time. The cheapest S wins, the smaller on a tie.
  (void)t;
  const long long tiles = (n + 127) / 128, chunks = (k + proj::kChunk - 1) / proj::kChunk;
  if (sms < 1) sms = 1;
  int best = 1;
  long long best_cost = -1;
  for (int s = 1; s <= kProjMaxSplits && s <= chunks && s <= sms; ++s) {
    const long long clusters = sms / s;
    const long long cost = (tiles + clusters - 1) / clusters * ((chunks + s - 1) / s) + 4;
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

int32_t proj_launch(const ProjLaunch& L, void* stream_handle) {
  using namespace proj;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_handle);
  if (!L.x || !L.w || !L.out) return TQ_ERR_INVALID_ARGUMENT;
  if (L.t < 1 || L.t > kMaxTokens || L.k % 8 || L.k < kChunk || L.n < 4 || L.n % 4 ||
      L.splits < 0 || L.splits > kProjMaxSplits)
    return TQ_ERR_UNSUPPORTED;
  const int tpad = (L.t + 15) / 16 * 16;
  const int stages = stages_for(tpad);
  if (stages < 2) return TQ_ERR_UNSUPPORTED;
  const int chunks = (L.k + kChunk - 1) / kChunk;
  const int tiles = (L.n + 127) / 128;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return TQ_ERR_CUDA;
  int splits = L.splits ? L.splits : proj_splits(L.n, L.k, L.t, sms);
  if (splits > chunks) splits = chunks;
  CUtensorMap tw, tx;
  if (!encode_rows(&tw, L.w, uint64_t(L.n), uint64_t(L.k), 128) ||
      !encode_rows(&tx, L.x, uint64_t(L.t), uint64_t(L.k), uint32_t(tpad)))
    return TQ_ERR_CUDA;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    for (int s = 1; s <= kProjMaxSplits && attr == cudaSuccess; ++s)
      attr = cudaFuncSetAttribute(kernel_for(s), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  int(kSmemBudget));
  });
  if (attr != cudaSuccess) return TQ_ERR_CUDA;
  // Persistent: as many clusters as fit at once (every cluster then runs from the start), at
  // most one per tile.
  int clusters = max_clusters(dev, splits, tpad);
  if (clusters < 1) return TQ_ERR_UNSUPPORTED;
  if (clusters > tiles) clusters = tiles;
  Args a;
  a.n = L.n;
  a.k = L.k;
  a.t = L.t;
  a.tpad = tpad;
  a.chunks = chunks;
  a.stages = stages;
  a.splits = splits;
  a.tiles = tiles;
  a.out = L.out;
  a.flags = L.flags;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(clusters * splits), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_for(tpad);
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = unsigned(splits);
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kernel_for(splits), tw, tx, a) != cudaSuccess) return TQ_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? TQ_OK : TQ_ERR_CUDA;
}

}  // namespace tq
