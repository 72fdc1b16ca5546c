// Compile-time layout of the paged MLA kernel: shared-memory map, TMEM columns, barriers.
//
// One CTA pair (a cluster of two, one CTA per SM) processes one query token at a time against a
// range of 64-row KV pages. CTA rank r owns
//   - the K-slice of QK^T: dims [256r, 256r+256) of the latent part (query slice held in TMEM),
//     plus dims [512+32r, +32) of the RoPE part for 576-wide rows (query slice in shared memory);
//   - the V-slice of PV and of the output: dims [256r, 256r+256).
// Each CTA sends its partial score tile (all 128 heads) to the peer with asynchronous remote
// stores that complete on the peer's mbarrier, and adds the peer's tile to its own. f32 addition is commutative, so both CTAs hold
// bit-identical scores and compute bit-identical softmax statistics and probabilities; each then
// runs PV for its half of the value dimension. Two softmax warpgroups split each page's 64 keys.
#pragma once

#include <cstdint>

namespace tq {
namespace mla {

constexpr int kPageRows = 64;
constexpr int kHeadsTile = 128;  // UMMA M
constexpr int kValueDim = 512;
constexpr int kValueHalf = 256;  // per CTA
constexpr int kStages = 3;
constexpr int kSoftmaxGroups = 2;  // warpgroups splitting the 64 keys of a page
constexpr int kSoftmaxWarps = 4 * kSoftmaxGroups;
constexpr int kSoftmaxThreads = 32 * kSoftmaxWarps;
constexpr int kThreads = 64 + kSoftmaxThreads;  // warp 0 TMA, warp 1 MMA, then softmax
constexpr int kKeysPerGroup = kPageRows / kSoftmaxGroups;  // 32

// Shared memory (byte offsets from a 1024-aligned base).
constexpr uint32_t kSmQRope = 0;             // [128 rows x 64 B], 64B swizzle
constexpr uint32_t kSmKv = 8192;             // kStages x stage
constexpr uint32_t kKvChunkBytes = 8192;     // [64 rows x 128 B], 128B swizzle
constexpr uint32_t kKvRopeOffset = 32768;    // [64 rows x 64 B] inside a stage
constexpr uint32_t kKvRopeBytes = 4096;
constexpr uint32_t kStageBytes = 36864;
// Partial-score tiles received from the peer, f32, double-buffered by page parity. A tile is
// [group][lane quarter][8 chunks][32 lanes][16 B]: each softmax warp owns one 4 KB block holding
// its 32 rows x 32 keys, chunk-major, so that a warp's store or load of one chunk touches 512
// contiguous bytes.
constexpr uint32_t kTileBytes = 32768;
constexpr uint32_t kGroupTileBytes = kTileBytes / kSoftmaxGroups;
constexpr uint32_t kWarpTileBytes = kGroupTileBytes / 4;
constexpr uint32_t kSmXbuf = kSmKv + kStages * kStageBytes;  // [2] tiles
constexpr uint32_t kSmRowMax = kSmXbuf + 2 * kTileBytes;      // f32 [2 parity][groups][128]
constexpr uint32_t kSmRowSum = kSmRowMax + 2 * kSoftmaxGroups * kHeadsTile * 4;  // f32 [groups][128]
constexpr uint32_t kSmBars = kSmRowSum + kSoftmaxGroups * kHeadsTile * 4;
constexpr int kNumBars = 25;
constexpr uint32_t kSmMisc = kSmBars + kNumBars * 8;  // tmem base holder, abort flag
constexpr uint32_t kSmUsed = kSmMisc + 16;
constexpr uint32_t kSmBytes = kSmUsed + 1024;          // slack for 1024-byte alignment

static_assert(kSmKv % 1024 == 0 && kStageBytes % 1024 == 0, "swizzle alignment");
static_assert(kSmXbuf % 1024 == 0, "tile alignment");
static_assert(kSmBars % 8 == 0, "mbarrier alignment");
static_assert(kSmBytes <= 232448, "shared memory per CTA");

// Barrier indices.
enum Bar : int {
  kBarKvFull = 0,                      // [kStages] TMA transaction barriers
  kBarKvEmpty = kBarKvFull + kStages,  // [kStages] PV done with the stage
  kBarQRopeFull = kBarKvEmpty + kStages,  // TMA of the RoPE query slice
  kBarQTmemFull,                       // latent query slice written to TMEM (one per group-0 warp)
  kBarQEmpty,                          // all QK MMAs of the segment done
  kBarSFull,                           // [2]
  kBarPFull = kBarSFull + 2,           // [2], one arrival per softmax warp
  kBarPvDone = kBarPFull + 2,          // [2]
  kBarOFull = kBarPvDone + 2,
  kBarOFree,                           // one arrival per softmax warp
  kBarXbFull,                          // [2] peer tile landed: armed locally with 32 KB expected
  kBarXbFree = kBarXbFull + 2,         // [2] peer consumed my tile: one remote arrival per peer warp
  kBarRowMax = kBarXbFree + 2,         // [2] both groups' partial row maxima written (per warp)
  kBarRowSum = kBarRowMax + 2,         // both groups' partial row sums written (per warp)
  kBarDrain,
  kBarCount
};
static_assert(kBarCount == kNumBars, "barrier count");

// TMEM columns (512 allocated).
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0;     // [2] x 64 columns: f32 scores, then bf16 P in the first 32
constexpr uint32_t kTmemQ = 128;   // 128 columns: latent query slice, bf16 pairs (A operand)
constexpr uint32_t kTmemO = 256;   // 256 columns of f32 output half

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
