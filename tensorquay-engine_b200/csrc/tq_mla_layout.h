// Compile-time layout of the paged MLA kernel: shared-memory map, TMEM columns, barriers.
//
// One CTA pair (a cluster of two, one CTA per SM) processes one query token at a time against a
// range of 64-row KV pages. CTA rank r owns
//   - the K-slice of QK^T: dims [256r, 256r+256) of the latent part, plus dims [512+32r, +32) of
//     the RoPE part for 576-wide rows;
//   - the V-slice of PV and of the output: dims [256r, 256r+256);
//   - the softmax of heads [64r, 64r+64).
// The two partial score tiles are summed through distributed shared memory, and the owner of a
// head sends its bf16 probabilities to the peer, so both halves of O see the same P.
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
constexpr int kOwnedRows = 64;

// Shared memory (byte offsets from a 1024-aligned base).
constexpr uint32_t kSmQMain = 0;             // 4 chunks x [128 rows x 128 B], 128B swizzle
constexpr uint32_t kQChunkBytes = 16384;
constexpr uint32_t kSmQRope = 65536;         // [128 rows x 64 B], 64B swizzle
constexpr uint32_t kSmKv = 73728;            // kStages x stage
constexpr uint32_t kKvChunkBytes = 8192;     // [64 rows x 128 B]
constexpr uint32_t kKvRopeOffset = 32768;    // [64 rows x 64 B] inside a stage
constexpr uint32_t kKvRopeBytes = 4096;
constexpr uint32_t kStageBytes = 36864;
constexpr uint32_t kSmXbuf = kSmKv + kStages * kStageBytes;  // peer partial scores, f32
constexpr uint32_t kXRowBytes = 272;                         // 256 B + 16 B pad (bank spread)
constexpr uint32_t kSmPrx = kSmXbuf + kOwnedRows * kXRowBytes;  // peer probabilities, bf16
constexpr uint32_t kPRowBytes = 144;                            // 128 B P + f32 correction + pad
constexpr uint32_t kSmStats = kSmPrx + kOwnedRows * kPRowBytes; // peer (1/l, lse)
constexpr uint32_t kSmBars = kSmStats + kOwnedRows * 8;
constexpr int kNumBars = 25;
constexpr uint32_t kSmMisc = kSmBars + kNumBars * 8;  // tmem base holder, abort flag
constexpr uint32_t kSmUsed = kSmMisc + 16;
constexpr uint32_t kSmBytes = kSmUsed + 1024;          // slack for 1024-byte alignment

static_assert(kSmXbuf % 16 == 0 && kSmPrx % 16 == 0 && kSmStats % 16 == 0, "alignment");
static_assert(kSmBars % 8 == 0, "mbarrier alignment");
static_assert(kSmBytes <= 232448, "shared memory per CTA");

// Barrier indices.
enum Bar : int {
  kBarKvFull = 0,                  // [kStages] TMA transaction barriers
  kBarKvEmpty = kBarKvFull + kStages,  // [kStages] PV done with the stage
  kBarQFull = kBarKvEmpty + kStages,
  kBarQEmpty,
  kBarSFull,                       // [2]
  kBarSFree = kBarSFull + 2,       // [2], 128 arrivals
  kBarPFull = kBarSFree + 2,       // [2], 128 arrivals
  kBarPvDone = kBarPFull + 2,      // [2]
  kBarOFull = kBarPvDone + 2,
  kBarOFree,                       // 128 arrivals
  kBarXbFull,                      // 64 remote arrivals: peer partial scores landed
  kBarXbFree,                      // 64 remote arrivals: peer consumed my partial scores
  kBarPrFull,                      // 64 remote arrivals: peer probabilities landed
  kBarPrFree,                      // 64 remote arrivals: peer consumed my probabilities
  kBarStFull,                      // 64 remote arrivals: peer row statistics landed
  kBarStFree,                      // 64 remote arrivals: peer consumed my statistics
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
