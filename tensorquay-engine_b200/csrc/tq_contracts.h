// Internal declarations shared by the host validation (tq_contracts.cpp) and the CUDA launch
// glue (tq_mla_kernels.cu). The public ABI is include/tq_mla.h.
//
// Generalisations of SmlaParams::new (crates/tq-core/src/contracts.rs:437-493) for the dense
// paged path:
//   - row format TQ_KV_BF16_ROPE576 (1152-byte rows); q is [T, H, 576] for it, out [T, H, 512];
//   - heads in {16, 32, 64, 128} (the reference accepts {32, 64});
//   - softmax scale: exactly 0.0625f for the reference's 512-wide formats (contracts.rs:446),
//     any finite positive f32 for TQ_KV_BF16_ROPE576;
//   - no idx / k_len tensors: dense attention over [0, min(kv_len, q_pos + 1));
//   - out may be f32 (a partial result merged later by tq_mla_combine);
//   - prefill plans (tq_mla_prefill_validate) have no 4-queries-per-sequence limit.
#pragma once

#include <cstddef>
#include <cstdint>

#include "../../include/tq_mla.h"

namespace tq {

bool params_intact(const TqMlaParams* p);
int32_t prologue_validate(const TqPrologueSpec* spec, TqContractError* err);
void philox_block(const uint32_t counter[4], const uint32_t key[2], uint32_t out[4]);
int32_t philox_words(uint64_t seed, uint64_t stream, uint64_t start, uint32_t* out,
                     uint64_t count);
float philox_uniform_f32(uint32_t word);

// Exchange region of the peer-memory context merge (tq_peer_merge.cu): a 256-byte header of u32
// words, then f32 partial out [T, H, 512] and f32 lse [T, H].
constexpr int kPeerMaxRanks = 8;
constexpr int kPeerHdrStep = 0;     // this rank's merge counter (device-side, graph-replayable)
constexpr int kPeerHdrError = 1;    // sticky device error flags (TQ_DEV_WAIT_TIMEOUT)
constexpr int kPeerHdrBlocks = 2;   // blocks of the running merge that have finished
constexpr int kPeerHdrReady = 16;   // [kPeerMaxRanks] rank r's partials of step k: k + 1
constexpr int kPeerHdrDone = 32;    // [kPeerMaxRanks] rank r has read them: k + 1
constexpr uint64_t kPeerHeaderBytes = 256;

struct PeerMergeLaunch {
  const uint8_t* regions[kPeerMaxRanks];  // every rank's region as mapped on this device
  int nranks, rank;
  uint64_t tokens, heads;
  uint8_t* out;
  float* lse;
  uint64_t out_stride_token, out_stride_head;
  int out_bf16;
};
int32_t peer_merge_launch(const PeerMergeLaunch& launch, void* stream);

// Weight-streaming projection out[T, N] = bf16(x[T, K] . w[N, K]^T) for T <= 128 tokens
// (tq_proj.cu): K split over the `splits` CTAs of a cluster per 128-row weight tile, their f32
// partial tiles added in split order through distributed shared memory.
struct ProjLaunch {
  const uint16_t* x;  // bf16 [T, K], packed
  const uint16_t* w;  // bf16 [N, K], packed
  int t, k, n;
  int splits;         // K splits (CTAs of one cluster), 1 to kProjMaxSplits; 0 picks them
  uint16_t* out;      // bf16 [T, N]
  int* flags;         // device error flags, may be null
};
constexpr int kProjMaxTokens = 128;
constexpr int kProjMaxSplits = 8;
// The K split of an N x K projection that balances the weight bytes over `sms` SMs.
int proj_splits(int n, int k, int t, int sms);
int32_t proj_launch(const ProjLaunch& launch, void* stream);

}  // namespace tq
