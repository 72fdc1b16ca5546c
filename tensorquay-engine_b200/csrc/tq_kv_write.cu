// KV cache writer: new latent rows into the paged pool (docs/DEV-PLAN.md:116, "latent -> 528 B KV
// writer"; row formats docs/HOST-CONTRACTS.md:122-123; paged addressing contracts.rs:182-209).
//
// One warp per row, grid-stride over the rows. A bf16 row (1024 or 1152 bytes) is copied with
// 16-byte loads and stores. An FP8 row is quantized on the way: lane l holds values
// [16 l, 16 l + 16) (two 16-byte loads of bf16), the eight lanes of a 128-value tile reduce their
// amax and NaN flag with shuffles, and each lane writes its 16 E4M3 codes as one 16-byte store;
// the first lane of a tile writes the tile's f32 scale after the 512 codes. The path is HBM-bound
// (1024 B read and 528 B written per FP8 row; 2 x 1152 B per 576-wide bf16 row).
//
// FP8 rule per tile (the reference defines none; this library's definition): a NaN in the tile
// gives scale NaN and codes 0x7F; amax == 0 gives scale 0 and codes 0; otherwise
// scale = amax / 448, inv = 448 / amax and code = E4M3(x * inv), or E4M3(x / scale) when inv
// overflows (amax below ~1.3e-36). f32 operations are IEEE round-to-nearest-even with subnormals
// kept (__fdiv_rn, __fmul_rn; no flush to zero); the conversion rounds to nearest even and
// saturates (cvt.rn.satfinite.e4m3x2.f32). One division per lane and tile, not per value: the
// per-value IEEE division made the writer compute-bound.

#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "tq_contracts.h"

namespace tq {
namespace kvw {

constexpr int kRowsPerBlock = 8;  // one warp per row
constexpr int kPageRows = 64;

struct Args {
  const uint8_t* src;
  long long src_stride;  // bytes between source rows
  uint8_t* kv;
  long long row_stride;  // bytes between pool rows
  long long pages;
  const int* page_table;
  long long sequences, slots;
  const int* seq_id;
  const int* pos;
  long long rows;
  int* flags;  // device error flags (may be null)
  const uint16_t* norm_w;  // RMSNorm weight, bf16 [512], or null
  float norm_eps;
};

__device__ __forceinline__ void flag(const Args& a, int bit) {
  if (a.flags) atomicOr(a.flags, bit);
}

// Two f32 values as E4M3 codes: `lo` in bits 0-7, `hi` in bits 8-15.
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Pool row of new row t, or null (flagged) when its sequence, position or page is out of range.
__device__ __forceinline__ uint8_t* slot_of(const Args& a, long long t, int lane) {
  const int s = a.seq_id[t], p = a.pos[t];
  if (s < 0 || s >= a.sequences) {
    if (lane == 0) flag(a, TQ_DEV_SEQ_RANGE);
    return nullptr;
  }
  if (p < 0 || p / kPageRows >= a.slots) {
    if (lane == 0) flag(a, TQ_DEV_TABLE_SHORT);
    return nullptr;
  }
  const int page = a.page_table[(long long)s * a.slots + p / kPageRows];
  if (page < 0 || page >= a.pages) {
    if (lane == 0) flag(a, TQ_DEV_PAGE_RANGE);
    return nullptr;
  }
  return a.kv + ((long long)page * kPageRows + p % kPageRows) * a.row_stride;
}

// One FP8 row: this lane's 16 values (two 16-byte words of bf16) to 16 codes, plus its tile's
// scale from the lane that starts the tile. All 32 lanes take part (shuffles).
__device__ __forceinline__ void quantize_store(uint8_t* dst, const uint4 w0, const uint4 w1,
                                               int lane) {
  const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  float x[16];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    x[2 * i] = __uint_as_float(words[i] << 16);
    x[2 * i + 1] = __uint_as_float(words[i] & 0xFFFF0000u);
  }
  // |x| as bf16 bit patterns order like the values, and every NaN pattern (above 0x7F80) is
  // larger than +inf's: one packed 16-bit unsigned max gives the tile's amax and its NaN test.
  uint32_t m = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i) m = __vmaxu2(m, words[i] & 0x7FFF7FFFu);
  // The eight lanes of a tile are aligned groups of eight: xor 1, 2, 4 stays inside one.
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) m = __vmaxu2(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  const uint32_t amax_bits = max(m & 0xFFFFu, m >> 16);
  const bool nan = amax_bits > 0x7F80u;
  const float amax = __uint_as_float(amax_bits << 16);
  float scale;
  uint4 codes;
  if (nan) {
    scale = __uint_as_float(0x7FC00000u);
    codes = make_uint4(0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
  } else if (amax == 0.f) {
    scale = 0.f;
    codes = make_uint4(0u, 0u, 0u, 0u);
  } else {
    scale = __fdiv_rn(amax, 448.f);
    const float inv = __fdiv_rn(448.f, amax);
    uint32_t c[8];
    if (inv != __uint_as_float(0x7F800000u)) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        c[i] = e4m3x2(__fmul_rn(x[2 * i], inv), __fmul_rn(x[2 * i + 1], inv));
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        c[i] = e4m3x2(__fdiv_rn(x[2 * i], scale), __fdiv_rn(x[2 * i + 1], scale));
    }
    codes = make_uint4(c[0] | (c[1] << 16), c[2] | (c[3] << 16), c[4] | (c[5] << 16),
                       c[6] | (c[7] << 16));
  }
  if (dst) {
    reinterpret_cast<uint4*>(dst)[lane] = codes;
    if ((lane & 7) == 0) reinterpret_cast<float*>(dst + 512)[lane >> 3] = scale;
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// RMSNorm of one row's 512 latent values, this lane holding values [16 lane, 16 lane + 16) as
// two 16-byte words of bf16 (in place). Only IEEE round-to-nearest f32 operations, in a fixed
// order: the lane's squares added in dim order, the 32 lane sums combined pairwise at distances
// 16, 8, 4, 2, 1 (both lanes of a pair get the same sum), mean = sum / 512, r = 1 / sqrt(mean +
// eps), y = bf16(bf16(x * r) * w): the normalised value is rounded to bf16 before the weight
// multiplies it, as the model's RMSNorm does (weight * hidden.to(bf16), modeling_glm5_next.py
// lines 77-81). All 32 lanes take part.
__device__ __forceinline__ void rms_norm_16(uint4& w0, uint4& w1, const uint16_t* nw, float eps,
                                            int lane) {
  uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float lo = __uint_as_float(words[i] << 16), hi = __uint_as_float(words[i] & 0xFFFF0000u);
    acc = __fadd_rn(acc, __fmul_rn(lo, lo));
    acc = __fadd_rn(acc, __fmul_rn(hi, hi));
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, o));
  const float r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, 512.f), eps)));
  const uint4 g0 = __ldg(reinterpret_cast<const uint4*>(nw) + 2 * lane);
  const uint4 g1 = __ldg(reinterpret_cast<const uint4*>(nw) + 2 * lane + 1);
  const uint32_t gw[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float lo = __uint_as_float(words[i] << 16), hi = __uint_as_float(words[i] & 0xFFFF0000u);
    const float wl = __uint_as_float(gw[i] << 16), wh = __uint_as_float(gw[i] & 0xFFFF0000u);
    const uint32_t n = pack_bf16x2(__fmul_rn(lo, r), __fmul_rn(hi, r));
    words[i] = pack_bf16x2(__fmul_rn(__uint_as_float(n << 16), wl),
                           __fmul_rn(__uint_as_float(n & 0xFFFF0000u), wh));
  }
  w0 = make_uint4(words[0], words[1], words[2], words[3]);
  w1 = make_uint4(words[4], words[5], words[6], words[7]);
}

template <int kFormat>
__global__ void __launch_bounds__(32 * kRowsPerBlock) kv_write_kernel(Args a) {
  const int lane = threadIdx.x & 31;
  const long long step = (long long)gridDim.x * kRowsPerBlock;
  const long long first = (long long)blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
  if constexpr (kFormat != TQ_KV_FP8_E4M3) {
    constexpr int kUnits = (kFormat == TQ_KV_BF16_ROPE576 ? 1152 : 1024) / 16;
    for (long long t = first; t < a.rows; t += step) {
      uint8_t* dst = slot_of(a, t, lane);
      if (!dst) continue;
      const uint8_t* src = a.src + t * a.src_stride;
      if (a.norm_w) {
        // Latent values normalised (this lane: units 2 lane, 2 lane + 1); RoPE units copied.
        uint4 w0 = __ldg(reinterpret_cast<const uint4*>(src) + 2 * lane);
        uint4 w1 = __ldg(reinterpret_cast<const uint4*>(src) + 2 * lane + 1);
        rms_norm_16(w0, w1, a.norm_w, a.norm_eps, lane);
        reinterpret_cast<uint4*>(dst)[2 * lane] = w0;
        reinterpret_cast<uint4*>(dst)[2 * lane + 1] = w1;
        if (kUnits > 64 && lane < kUnits - 64)
          reinterpret_cast<uint4*>(dst)[64 + lane] =
              __ldg(reinterpret_cast<const uint4*>(src) + 64 + lane);
        continue;
      }
#pragma unroll
      for (int i = lane; i < kUnits; i += 32)
        reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
    }
  } else {
    // Two rows per warp and iteration: both rows' loads are in flight before either converts.
    for (long long t = first; t < a.rows; t += 2 * step) {
      const long long t2 = t + step;
      const bool has2 = t2 < a.rows;
      const uint4* s1 = reinterpret_cast<const uint4*>(a.src + t * a.src_stride) + 2 * lane;
      uint4 a0 = __ldg(s1), a1 = __ldg(s1 + 1);
      uint4 b0 = make_uint4(0u, 0u, 0u, 0u), b1 = b0;
      if (has2) {
        const uint4* s2 = reinterpret_cast<const uint4*>(a.src + t2 * a.src_stride) + 2 * lane;
        b0 = __ldg(s2);
        b1 = __ldg(s2 + 1);
      }
      if (a.norm_w) {  // quantize the normalised bf16 values
        rms_norm_16(a0, a1, a.norm_w, a.norm_eps, lane);
        if (has2) rms_norm_16(b0, b1, a.norm_w, a.norm_eps, lane);
      }
      quantize_store(slot_of(a, t, lane), a0, a1, lane);
      if (has2) quantize_store(slot_of(a, t2, lane), b0, b1, lane);
    }
  }
}

int sm_count(int device) {
  static std::mutex mu;
  static int cached[128] = {0};
  if (device < 0 || device >= 128) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[device]) return cached[device];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  cached[device] = n;
  return n;
}

}  // namespace kvw
}  // namespace tq

extern "C" int32_t tq_kv_write(const TqKvWriteSpec* spec, int32_t* device_flags, void* stream,
                               TqContractError* err) {
  using namespace tq::kvw;
  const int32_t st = tq_kv_write_validate(spec, err);
  if (st != TQ_OK) return st;
  const TqKvWriteSpec& s = *spec;
  const long long rows = (long long)s.src.shape[0];
  if (rows == 0) return TQ_OK;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) {
    if (err) { err->field = "device"; err->kind = TQ_ERR_CUDA; }
    return TQ_ERR_CUDA;
  }
  const int sms = sm_count(device);
  if (sms <= 0) {
    if (err) { err->field = "device"; err->kind = TQ_ERR_CUDA; }
    return TQ_ERR_CUDA;
  }
  Args a;
  a.src = reinterpret_cast<const uint8_t*>(s.src.device_address);
  a.src_stride = (long long)s.src.strides_bytes[0];
  a.kv = reinterpret_cast<uint8_t*>(s.kv.device_address);
  a.row_stride = (long long)s.kv.strides_bytes[1];
  a.pages = (long long)s.kv.shape[0];
  a.page_table = reinterpret_cast<const int*>(s.page_table.device_address);
  a.sequences = (long long)s.page_table.shape[0];
  a.slots = (long long)s.page_table.shape[1];
  a.seq_id = reinterpret_cast<const int*>(s.seq_id.device_address);
  a.pos = reinterpret_cast<const int*>(s.pos.device_address);
  a.rows = rows;
  a.flags = device_flags;
  a.norm_w = s.norm_weight.rank != 0 ? reinterpret_cast<const uint16_t*>(s.norm_weight.device_address)
                                     : nullptr;
  a.norm_eps = s.norm_eps;
  const long long want = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
  const int blocks = int(want < 8ll * sms ? want : 8ll * sms);
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  switch (s.kv_format) {
    case TQ_KV_BF16: kv_write_kernel<TQ_KV_BF16><<<blocks, 32 * kRowsPerBlock, 0, cs>>>(a); break;
    case TQ_KV_FP8_E4M3:
      kv_write_kernel<TQ_KV_FP8_E4M3><<<blocks, 32 * kRowsPerBlock, 0, cs>>>(a);
      break;
    default:
      kv_write_kernel<TQ_KV_BF16_ROPE576><<<blocks, 32 * kRowsPerBlock, 0, cs>>>(a);
      break;
  }
  if (cudaGetLastError() != cudaSuccess) {
    if (err) { err->field = "launch"; err->kind = TQ_ERR_CUDA; }
    return TQ_ERR_CUDA;
  }
  if (err) { err->field = nullptr; err->kind = TQ_OK; }
  return TQ_OK;
}
