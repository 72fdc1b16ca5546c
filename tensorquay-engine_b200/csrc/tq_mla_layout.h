// Compile-time layout of the paged MLA kernel: shared-memory map, TMEM columns, barriers.
//
// One CTA pair (a cluster of two, one CTA per SM) processes one query token at a time against a
// range of 64-row KV pages. CTA rank r owns
//   - the keys [32r, 32r + 32) of every page for QK^T and the softmax: S_r = Q K_r^T over the
//     full query width (M = 128 heads, N = 32 keys), with the query's first 384 dims in TMEM
//     and the rest in shared memory;
//   - the value dims [256r, 256r + 256) for PV and the output: O_r += P V[:, 256r:256r+256]
//     over all 64 keys, its own keys' P from TMEM and the peer's P from shared memory.
// Per page the CTAs exchange only bf16 probabilities and one f32 reference maximum per head
// row (8.5 KB each way), pushed with asynchronous remote stores that complete on the receiver's
// mbarrier. Both CTAs derive the same running maximum, so the two halves of O share one
// normalisation.
#pragma once

#include <cstdint>

namespace tq {
namespace mla {

constexpr int kPageRows = 64;
constexpr int kKeysPerCta = 32;
constexpr int kHeadsTile = 128;  // UMMA M
constexpr int kValueDim = 512;
constexpr int kValueHalf = 256;  // per CTA
constexpr int kStages = 3;
// Scheduling cost of starting a segment (a token's page range on one CTA pair: query load,
// pipeline refill, epilogue), in pages. The partition balances pages + this per segment.
constexpr int kSegmentCostPages = 8;
constexpr int kSoftmaxWarps = 4;
constexpr int kSoftmaxThreads = 32 * kSoftmaxWarps;
constexpr int kThreads = 64 + kSoftmaxThreads;  // warp 0 TMA, warp 1 MMA, warps 2-5 softmax
constexpr int kConvertWarps = 4;                 // FP8 rows, sparse plans: warps 6-9 fill the pages
constexpr int kThreadsGather = kThreads + 32 * kConvertWarps;
constexpr int kFp8RowCodes = 512;                // E4M3 codes per row, then 4 f32 scales
constexpr int kQTmemDims = 384;                 // query dims held in TMEM (A operand)

// Shared memory (byte offsets from a 1024-aligned base).
// Query dims [384, width): up to 3 chunks of [128 rows x 64 dims] bf16, 128B swizzle.
constexpr uint32_t kSmQ = 0;
constexpr uint32_t kQChunkBytes = 16384;
constexpr uint32_t kSmKv = 3 * kQChunkBytes;
// A stage holds one page: this CTA's 32 keys x all 64-dim chunks (up to 9), then the peer's 32
// keys x this CTA's 4 value chunks, both as [8-key group][chunk][8 keys x 128 B] (128B swizzle):
// 1 KB atoms, chunks 1 KB apart, key groups (chunks x 1 KB) apart.
constexpr uint32_t kAtomBytes = 1024;
constexpr uint32_t kKvChunkBytes = 4096;  // one chunk of 32 keys
constexpr int kQkChunksMax = 9;
constexpr uint32_t kPvxOffset = kQkChunksMax * kKvChunkBytes;
constexpr uint32_t kStageBytes = kPvxOffset + 4 * kKvChunkBytes;
// Peer probabilities, double-buffered by page parity: bf16 [4 key chunks][128 rows][8 keys]
// (no-swizzle K-major UMMA layout: 8-row groups 128 B apart, key chunks 2 KB apart), then the
// peer's f32 reference maximum per row.
constexpr uint32_t kPChunkBytes = 2048;
constexpr uint32_t kPBytes = 4 * kPChunkBytes;
constexpr uint32_t kPMsgBytes = kPBytes + kHeadsTile * 4;
constexpr uint32_t kSmPeer = kSmKv + kStages * kStageBytes;
constexpr uint32_t kSmLsum = kSmPeer + 2 * kPMsgBytes;  // peer's f32 row sums
constexpr uint32_t kSmBars = kSmLsum + kHeadsTile * 4;
constexpr int kNumBars = 46;
constexpr uint32_t kSmMisc = kSmBars + kNumBars * 8;  // tmem base holder, abort flag
// FP8 rows: each convert warp's next-page scale quadruples (8 keys x 16 B); their codes wait in
// the query chunk that 512-wide queries leave unused.
constexpr uint32_t kSmFp8Scales = kSmMisc + 16;
constexpr uint32_t kSmUsed = kSmFp8Scales + 4 * 128;
constexpr uint32_t kSmBytes = kSmUsed + 1024;          // slack for 1024-byte alignment

// Bytes one softmax warp receives per page (its 32 rows of P and of the reference maximum).
constexpr uint32_t kWarpMsgBytes = 32 * 64 + 32 * 4;

static_assert(kSmKv % 1024 == 0 && kStageBytes % 1024 == 0, "swizzle alignment");
static_assert(kSmPeer % 128 == 0, "operand alignment");
static_assert(kSmBars % 8 == 0, "mbarrier alignment");
static_assert(kSmBytes <= 232448, "shared memory per CTA");

// Barrier indices.
enum Bar : int {
  kBarKvFull = 0,                       // [kStages] TMA transaction barriers
  kBarKvEmpty = kBarKvFull + kStages,   // [kStages] PV done with the stage
  kBarQSmemFull = kBarKvEmpty + kStages,  // TMA of the shared-memory query dims
  kBarQEmpty,                           // all QK MMAs of the segment done
  kBarSFull,                            // [2]
  kBarPFull = kBarSFull + 2,            // [2] both halves of P ready (one arrival per warp)
  kBarPvDone = kBarPFull + 2,           // [2]
  kBarOFull = kBarPvDone + 2,
  kBarOFree,                            // one arrival per softmax warp
  kBarMsgFull,                          // [2][4] peer warp's P rows + maxima landed (tx bytes)
  kBarMsgFree = kBarMsgFull + 8,        // [2] the peer's PV of the buffer's last page is done
                                        //     (one arrival, the peer MMA warp's commit)
  kBarLsumFull = kBarMsgFree + 2,       // [4] peer warp's row sums landed (tx bytes)
  kBarKvGrant = kBarLsumFull + 4,       // [kStages] FP8: a page's stage is free (the producer,
                                        //     the only waiter on kBarKvEmpty, passes it on)
  kBarPeerGrant = kBarKvGrant + kStages,  // [kStages] FP8: the peer's stage is free for this
                                        //     CTA's copy of its keys' value half (peer producer)
  kBarSpare = kBarPeerGrant + kStages,  // [15 - 2 kStages] unused
  kBarDrain = kBarSpare + 15 - 2 * kStages,
  kBarCount
};
static_assert(kBarCount == kNumBars, "barrier count");

// TMEM columns (512 allocated).
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0;    // [2] x 32 columns: f32 scores, then bf16 P in the first 16
constexpr uint32_t kTmemQ = 64;   // 192 columns: query dims [0, 384) as bf16 pairs (A operand)
constexpr uint32_t kTmemO = 256;  // 256 columns of f32 output half

// Workspace header words.
enum Header : int {
  kHdrError = 0,
  kHdrTotalPages = 1,
  kHdrQuota = 2,
  kHdrNumCombine = 3,
  kHdrNumEmpty = 4,
  kHdrPairs = 5,
  kHdrTokens = 6,
  kHdrTimeoutWhere = 8,  // role << 24 | page counter, bit 30 set (0 = no timeout)
  kHdrTimeoutBar = 9,    // barrier index | parity << 16
  kHdrTimeoutCta = 10,   // blockIdx.x * 1024 + threadIdx.x
  kHdrWords = 16
};

}  // namespace mla
}  // namespace tq
