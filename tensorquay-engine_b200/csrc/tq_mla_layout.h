// Compile-time layout of the paged MLA kernel: shared-memory map, TMEM columns, barriers.
//
// One CTA pair (a cluster of two, one CTA per SM) processes one query token at a time against a
// range of 64-row KV pages. CTA rank r owns
//   - the K-slice of QK^T: dims [256r, 256r+256) of the latent part, plus dims [512+32r, +32) of
//     the RoPE part for 576-wide rows;
//   - the V-slice of PV and of the output: dims [256r, 256r+256).
// Each CTA sends its partial score tile (all 128 heads) to the peer through distributed shared
// memory and adds the peer's tile to its own. f32 addition is commutative, so both CTAs hold
// bit-identical scores and compute bit-identical softmax statistics and probabilities; each then
// runs PV for its half of the value dimension.
#pragma once

#include <cstdint>

namespace tq {
namespace mla {

constexpr int kPageRows = 64;
constexpr int kHeadsTile = 128;  // UMMA M
constexpr int kValueDim = 512;
constexpr int kValueHalf = 256;  // per CTA
constexpr int kStages = 3;
constexpr int kThreads = 192;    // warp 0 TMA, warp 1 MMA, warps 2-5 softmax/epilogue
constexpr int kSoftmaxThreads = 128;
constexpr int kSoftmaxWarps = 4;

// Shared memory (byte offsets from a 1024-aligned base).
constexpr uint32_t kSmQMain = 0;             // 4 chunks x [128 rows x 128 B], 128B swizzle
constexpr uint32_t kQChunkBytes = 16384;
constexpr uint32_t kSmQRope = 65536;         // [128 rows x 64 B], 64B swizzle
constexpr uint32_t kSmKv = 73728;            // kStages x stage
constexpr uint32_t kKvChunkBytes = 8192;     // [64 rows x 128 B]
constexpr uint32_t kKvRopeOffset = 32768;    // [64 rows x 64 B] inside a stage
constexpr uint32_t kKvRopeBytes = 4096;
constexpr uint32_t kStageBytes = 36864;
// Peer partial scores, f32 [128 rows x 64 keys]; 16-byte chunk k of row h is stored at chunk
// k ^ (h & 7) so that eight consecutive rows read eight different bank groups.
constexpr uint32_t kSmXbuf = kSmKv + kStages * kStageBytes;
constexpr uint32_t kXRowBytes = 256;
constexpr uint32_t kSmBars = kSmXbuf + kHeadsTile * kXRowBytes;
constexpr int kNumBars = 21;
constexpr uint32_t kSmMisc = kSmBars + kNumBars * 8;  // tmem base holder, abort flag
constexpr uint32_t kSmUsed = kSmMisc + 16;
constexpr uint32_t kSmBytes = kSmUsed + 1024;          // slack for 1024-byte alignment

static_assert(kSmXbuf % 1024 == 0, "alignment");
static_assert(kSmBars % 8 == 0, "mbarrier alignment");
static_assert(kSmBytes <= 232448, "shared memory per CTA");

// Barrier indices.
enum Bar : int {
  kBarKvFull = 0,                  // [kStages] TMA transaction barriers
  kBarKvEmpty = kBarKvFull + kStages,  // [kStages] PV done with the stage
  kBarQFull = kBarKvEmpty + kStages,
  kBarQEmpty,
  kBarSFull,                       // [2]
  kBarSFree = kBarSFull + 2,       // [2], one arrival per softmax warp
  kBarPFull = kBarSFree + 2,       // [2], one arrival per softmax warp
  kBarPvDone = kBarPFull + 2,      // [2]
  kBarOFull = kBarPvDone + 2,
  kBarOFree,                       // one arrival per softmax warp
  kBarXbFull,                      // one remote arrival per peer softmax warp: its scores landed
  kBarXbFree,                      // one remote arrival per peer softmax warp: it read my scores
  kBarDrain,
  kBarCount
};
static_assert(kBarCount == kNumBars, "barrier count");

// TMEM columns (512 allocated).
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0;     // [2] x 64 columns of f32 scores
constexpr uint32_t kTmemP = 128;   // [2] x 32 columns of packed bf16 probabilities
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
  kHdrTimeoutBar = 9,    // barrier smem offset | parity << 16
  kHdrTimeoutCta = 10,   // blockIdx.x * 1024 + threadIdx.x
  kHdrWords = 16
};

}  // namespace mla
}  // namespace tq
