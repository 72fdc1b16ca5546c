// Context merge over NVLink peer memory: the LSE merge of a context split (decode context
// parallelism, docs/ARCHITECTURE.md:240-241,313) done by one kernel per rank that reads the
// other ranks' partial results directly from their memory, instead of an NCCL all-gather
// followed by a local merge.
//
// Every rank owns one exchange region (cudaMalloc, exported with CUDA IPC and opened by every
// other rank of the communicator):
//   header (256 B): step (this rank's merge counter), error flags, block counter,
//                   ready[r] and done[r] (u32 per rank, written by rank r over NVLink)
//   partials:       f32 out [T, H, 512], then f32 lse [T, H]
// Merge k (every rank calls it in the same order; k is this rank's device-side step counter):
//   1. block 0 publishes ready = k + 1 into every peer's header (a release store at system
//      scope, after griddepcontrol.wait, so the decode kernel's partials are visible to a peer
//      that acquires it);
//   2. every block waits until all peers' ready in its own header reach k + 1 (bounded);
//   3. blocks merge rows (t, h), four at a time: m = max lse, w_r = exp(lse_r - m), out = sum_r w_r o_r / sum w,
//      lse = m + ln sum w, reading the peers' rows over NVLink (L2-only loads);
//   4. the last block to finish publishes done = k + 1 into every peer's header, waits until
//      all peers' done reach k + 1 (they have read this rank's partials), and advances the step.
// The next decode on this stream may then overwrite the partials. All waits are bounded by
// the global timer and a poll count; a timeout sets TQ_DEV_WAIT_TIMEOUT in the header and the
// kernel returns without merging (the plan is then unusable, like a failed communicator).

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "tq_contracts.h"

namespace tq {
namespace peer {

constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s
constexpr uint32_t kMaxPolls = 1u << 26;

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Waits until every peer's counter in `flags` reaches `target`; false after the bound.
__device__ bool wait_all(const uint32_t* flags, int nranks, int rank, uint32_t target) {
  const uint64_t t0 = now_ns();
  for (uint32_t i = 0;; ++i) {
    bool all = true;
    for (int r = 0; r < nranks; ++r)
      if (r != rank && ld_acquire_sys(flags + r) < target) all = false;
    if (all) return true;
    if ((i & 255) == 255 && (now_ns() - t0 > kWaitNs || i > kMaxPolls)) return false;
    __nanosleep(64);
  }
}

struct Args {
  uint32_t* header;              // this rank's header (local)
  const uint8_t* regions[kPeerMaxRanks];  // every rank's region (this rank's own included)
  uint32_t* peer_headers[kPeerMaxRanks];  // every rank's header, as mapped here
  int nranks, rank;
  uint64_t rows;                 // T * H
  uint64_t heads;
  uint64_t out_offset, lse_offset;  // byte offsets of the partials in a region
  uint8_t* out;
  float* lse;
  uint64_t out_stride_token, out_stride_head;
  int out_bf16;
};

__global__ void __launch_bounds__(512) peer_merge_kernel(Args a) {
  // Launched as a programmatic dependent of the decode's last kernel: nothing is read or
  // published before that kernel's results are complete and visible.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  uint32_t* h = a.header;
  __shared__ uint32_t s_step;
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    s_step = *reinterpret_cast<volatile uint32_t*>(h + kPeerHdrStep);
    s_ok = *reinterpret_cast<volatile uint32_t*>(h + kPeerHdrError) == 0;
  }
  __syncthreads();
  const uint32_t k = s_step;
  if (!s_ok) return;  // an earlier timeout: the plan is unusable
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    // The decode's partials are complete and visible here (griddepcontrol.wait); the release
    // store orders them before the flag for a peer that acquires it.
    for (int r = 0; r < a.nranks; ++r)
      if (r != a.rank) st_release_sys(a.peer_headers[r] + kPeerHdrReady + a.rank, k + 1);
  }
  if (threadIdx.x == 0) {
    if (!wait_all(h + kPeerHdrReady, a.nranks, a.rank, k + 1)) {
      atomicOr(reinterpret_cast<int*>(h + kPeerHdrError), TQ_DEV_WAIT_TIMEOUT);
      s_ok = 0;
    }
  }
  __syncthreads();
  if (s_ok) {
    // Four rows at a time per block: 128 threads per row, 4 of its 512 values per thread.
    const int tr = threadIdx.x & 127, c = tr * 4;
    for (uint64_t row = blockIdx.x * 4ull + (threadIdx.x >> 7); row < a.rows;
         row += gridDim.x * 4ull) {
      // Every rank's lse and this thread's 4 values of the row, all loads in flight together.
      float lr[kPeerMaxRanks];
      float4 o[kPeerMaxRanks];
#pragma unroll
      for (int r = 0; r < kPeerMaxRanks; ++r) {
        if (r < a.nranks) {
          lr[r] = __ldcg(reinterpret_cast<const float*>(a.regions[r] + a.lse_offset) + row);
          o[r] = __ldcg(reinterpret_cast<const float4*>(a.regions[r] + a.out_offset +
                                                        row * 2048) + tr);
        }
      }
      float m = -INFINITY;
#pragma unroll
      for (int r = 0; r < kPeerMaxRanks; ++r)
        if (r < a.nranks) m = fmaxf(m, lr[r]);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      float wsum = 0.f;
      if (m != -INFINITY) {
#pragma unroll
        for (int r = 0; r < kPeerMaxRanks; ++r) {
          if (r >= a.nranks) continue;
          const float w = expf(lr[r] - m);
          if (w == 0.f) continue;  // a part with no keys (lse -inf) adds nothing
          acc.x += w * o[r].x;
          acc.y += w * o[r].y;
          acc.z += w * o[r].z;
          acc.w += w * o[r].w;
          wsum += w;
        }
      }
      const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
      const uint64_t t = row / a.heads, hh = row % a.heads;
      uint8_t* dst = a.out + t * a.out_stride_token + hh * a.out_stride_head;
      if (a.out_bf16) {
        uint32_t lo, hi;
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(acc.y * inv), "f"(acc.x * inv));
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(acc.w * inv), "f"(acc.z * inv));
        *reinterpret_cast<uint2*>(dst + c * 2) = make_uint2(lo, hi);
      } else {
        *reinterpret_cast<float4*>(dst + c * 4) =
            make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
      }
      if (tr == 0) a.lse[row] = wsum > 0.f ? m + logf(wsum) : -INFINITY;
    }
  }
  // The last block to finish tells every peer this rank has read its partials, then waits for
  // the same from every peer before the step advances.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t n = atomicAdd(h + kPeerHdrBlocks, 1u);
    if (n == gridDim.x - 1) {
      *reinterpret_cast<volatile uint32_t*>(h + kPeerHdrBlocks) = 0;
      // Every block's loads of peer memory returned before its fence and count above.
      for (int r = 0; r < a.nranks; ++r)
        if (r != a.rank) st_release_sys(a.peer_headers[r] + kPeerHdrDone + a.rank, k + 1);
      if (!wait_all(h + kPeerHdrDone, a.nranks, a.rank, k + 1))
        atomicOr(reinterpret_cast<int*>(h + kPeerHdrError), TQ_DEV_WAIT_TIMEOUT);
      *reinterpret_cast<volatile uint32_t*>(h + kPeerHdrStep) = k + 1;
    }
  }
}

}  // namespace peer

int32_t peer_merge_launch(const PeerMergeLaunch& L, void* stream_handle) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_handle);
  peer::Args a;
  a.header = reinterpret_cast<uint32_t*>(const_cast<uint8_t*>(L.regions[L.rank]));
  for (int r = 0; r < kPeerMaxRanks; ++r) {
    a.regions[r] = r < L.nranks ? L.regions[r] : nullptr;
    a.peer_headers[r] =
        r < L.nranks ? reinterpret_cast<uint32_t*>(const_cast<uint8_t*>(L.regions[r])) : nullptr;
  }
  a.nranks = L.nranks;
  a.rank = L.rank;
  a.rows = L.tokens * L.heads;
  a.heads = L.heads;
  a.out_offset = kPeerHeaderBytes;
  a.lse_offset = kPeerHeaderBytes + a.rows * 2048;
  a.out = L.out;
  a.lse = L.lse;
  a.out_stride_token = L.out_stride_token;
  a.out_stride_head = L.out_stride_head;
  a.out_bf16 = L.out_bf16;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return TQ_ERR_CUDA;
  const uint64_t quads = (a.rows + 3) / 4;
  const uint64_t want = quads < uint64_t(sms) ? quads : uint64_t(sms);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(want ? want : 1), 1, 1);
  cfg.blockDim = dim3(512, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, peer::peer_merge_kernel, a) != cudaSuccess) return TQ_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? TQ_OK : TQ_ERR_CUDA;
}

}  // namespace tq
