// MLA prologue: "q_a -> norm -> q_b -> absorb; kv_a -> norm -> cache write" (planned as one
// fused step in docs/DEV-PLAN.md:116; the key absorption is the q_abs = w_uk^T q of
// reference/src/tq_reference/mla_attention.py:150), for the no-RoPE rows of the reference's model
// (rope_dim 0, docs/research/glm-5.md:163-167) and for 576-wide rows (rope_dim 64).
//
// Per call (T tokens, Dr = rope_dim, W = 512 + Dr):
//   1. cq  = x . w_qa^T                 GEMM, bf16 in, f32 accumulate, bf16 out
//   2. cq <- bf16(rms(cq)) * q_norm     rms_rows_kernel (in place)
//   3. qf  = cq . w_qb^T                plain GEMM                       [T, H, Dn + Dr]
//   4. q[:, :, :512] = qf[:, :, :Dn] . w_uk[h]   one strided-batched GEMM over the heads, written
//                                       straight into q's row layout (ldc = H * W)
//   5. q[:, :, 512:] = rope(qf[:, :, Dn:]) and kvf[:, 512:] rotated in place (rope_rows_kernel)
//   6. kvf = x . w_kva^T                plain GEMM                       [T, W]
//   7. tq_kv_write: bf16(rms(kvf[:512])) * kv_norm and the row written (FP8 rows quantized) to the
//      token's pool slot through the page table
// Steps 6-7 (the cache branch) run on a per-device side stream, forked from the caller's stream
// by an event and joined back into it before the call returns, beside steps 1-4 (the query
// branch) on the caller's stream; step 5 follows on the side stream once q_b is written, beside
// the absorption. The pattern is graph-capturable.
// At decode sizes (T <= 128) the narrow projections (steps 1 and 6) run on tq_proj.cu's
// weight-streaming kernel; the other GEMMs are cuBLAS (opened at run time as libcublas.so.12: a
// process that already has it, e.g. through PyTorch, shares that copy); everything else is this
// library's kernels. At decode
// sizes the step is HBM-bound on the weights (w_qb and w_uk dominate). The q norm accumulates
// squares in f32; RoPE reduces its angle pos * theta^(-2i/64) in f64 before the sine and cosine,
// so positions up to 2^31 keep full precision.

#include <cublas_v2.h>
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "tq_contracts.h"

namespace tq {
namespace prologue {

constexpr int kRopeDim = 64;
constexpr int kLatent = 512;
constexpr uint64_t kCublasScratch = 32ull << 20;

// ------------------------------------------------------------------------------ cuBLAS, opened
struct Blas {
  cublasStatus_t (*create)(cublasHandle_t*);
  cublasStatus_t (*set_stream)(cublasHandle_t, cudaStream_t);
  cublasStatus_t (*set_workspace)(cublasHandle_t, void*, size_t);
  cublasStatus_t (*gemm)(cublasHandle_t, cublasOperation_t, cublasOperation_t, int, int, int,
                         const void*, const void*, cudaDataType, int, const void*, cudaDataType,
                         int, const void*, void*, cudaDataType, int, cublasComputeType_t,
                         cublasGemmAlgo_t);
  cublasStatus_t (*gemm_batched)(cublasHandle_t, cublasOperation_t, cublasOperation_t, int, int,
                                 int, const void*, const void*, cudaDataType, int, long long,
                                 const void*, cudaDataType, int, long long, const void*, void*,
                                 cudaDataType, int, long long, int, cublasComputeType_t,
                                 cublasGemmAlgo_t);
  bool ok = false;
};

const Blas* blas() {
  static Blas b;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libcublas.so.12", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libcublas.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    b.create = reinterpret_cast<decltype(b.create)>(dlsym(h, "cublasCreate_v2"));
    b.set_stream = reinterpret_cast<decltype(b.set_stream)>(dlsym(h, "cublasSetStream_v2"));
    b.set_workspace = reinterpret_cast<decltype(b.set_workspace)>(dlsym(h, "cublasSetWorkspace_v2"));
    b.gemm = reinterpret_cast<decltype(b.gemm)>(dlsym(h, "cublasGemmEx"));
    b.gemm_batched =
        reinterpret_cast<decltype(b.gemm_batched)>(dlsym(h, "cublasGemmStridedBatchedEx"));
    b.ok = b.create && b.set_stream && b.set_workspace && b.gemm && b.gemm_batched;
  });
  return b.ok ? &b : nullptr;
}

// One handle per device, created on the first call with that device current.
cublasHandle_t handle_for(int device) {
  static std::mutex mu;
  static cublasHandle_t cache[128] = {nullptr};
  const Blas* b = blas();
  if (!b || device < 0 || device >= 128) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[device]) {
    cublasHandle_t h = nullptr;
    if (b->create(&h) != CUBLAS_STATUS_SUCCESS) return nullptr;
    cache[device] = h;
  }
  return cache[device];
}

// ------------------------------------------------------------------------------ kernels
__device__ __forceinline__ float bf16_to_f32(uint16_t v) { return __uint_as_float(uint32_t(v) << 16); }

__device__ __forceinline__ uint16_t f32_to_bf16(float x) {
  uint16_t r;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(x));
  return r;
}

// Rows of `width` bf16 values (packed, `rows` of them): x <- bf16(bf16(x * r) * w), r = 1 /
// sqrt(mean of squares + eps), squares summed in f32; the normalised value is rounded to bf16
// before the weight multiplies it, as in the model's RMSNorm (weight * hidden.to(bf16)). One
// 256-thread block per row, grid-stride; a thread takes eight values at a time (16-byte loads
// and stores: width is a multiple of 8 and the rows and weights are 16-byte aligned).
__global__ void __launch_bounds__(256) rms_rows_kernel(uint16_t* x, int width, long long rows,
                                                       const uint16_t* __restrict__ w, float eps) {
  __shared__ float part[8];
  __shared__ float s_r;
  for (long long row = blockIdx.x; row < rows; row += gridDim.x) {
    uint16_t* v = x + row * width;
    float sq = 0.f;
    for (int i = threadIdx.x * 8; i < width; i += 256 * 8) {
      const uint4 p = *reinterpret_cast<const uint4*>(v + i);
      const uint32_t u[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float f0 = bf16_to_f32(uint16_t(u[k] & 0xFFFF)), f1 = bf16_to_f32(uint16_t(u[k] >> 16));
        sq += f0 * f0;
        sq += f1 * f1;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xFFFFFFFFu, sq, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int k = 0; k < 8; ++k) t += part[k];
      s_r = 1.f / sqrtf(t / float(width) + eps);
    }
    __syncthreads();
    const float r = s_r;
    for (int i = threadIdx.x * 8; i < width; i += 256 * 8) {
      const uint4 p = *reinterpret_cast<const uint4*>(v + i);
      const uint4 q = *reinterpret_cast<const uint4*>(w + i);
      const uint32_t u[4] = {p.x, p.y, p.z, p.w}, g[4] = {q.x, q.y, q.z, q.w};
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint16_t lo = f32_to_bf16(
            bf16_to_f32(f32_to_bf16(bf16_to_f32(uint16_t(u[k] & 0xFFFF)) * r)) *
            bf16_to_f32(uint16_t(g[k] & 0xFFFF)));
        const uint16_t hi = f32_to_bf16(
            bf16_to_f32(f32_to_bf16(bf16_to_f32(uint16_t(u[k] >> 16)) * r)) *
            bf16_to_f32(uint16_t(g[k] >> 16)));
        o[k] = uint32_t(lo) | (uint32_t(hi) << 16);
      }
      *reinterpret_cast<uint4*>(v + i) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    __syncthreads();  // part / s_r are reused by the next row
  }
}

// cos and sin of pair i of the 64 RoPE values at position `pos`: angle pos * theta^(-2i/64),
// reduced modulo 2 pi in f64.
__device__ __forceinline__ void rope_angle(int i, int pos, double log2_theta, float* c, float* s) {
  const double freq = exp2(-double(2 * i) / double(kRopeDim) * log2_theta);
  const double angle = fmod(double(pos) * freq, 6.283185307179586476925286766559);
  double sd, cd;
  sincos(angle, &sd, &cd);
  *c = float(cd);
  *s = float(sd);
}

// dst[r, 2i .. 2i + 1] = rope(src[r, 2i .. 2i + 1]) for the `per_token` rows r of each of
// `tokens` tokens (row r = t * per_token + j, position pos[t]), rows of 64 values at the given
// element offsets and row strides. Block (x, y) takes rows 64 y .. 64 y + 63 of tokens x,
// x + gridDim.x, ...: the first warp computes the token's 32 (cos, sin) pairs once into shared
// memory, then each warp rotates eight whole rows (all eight loaded before any is written), lane
// i pair i. Each lane reads its pairs before writing them, so src may equal dst (the kv RoPE
// slice is rotated in place). q: per_token H, src qf + Dn, dst q + 512; kv: per_token 1,
// src = dst = kvf + 512.
__global__ void __launch_bounds__(256) rope_rows_kernel(const uint16_t* src, long long src_stride,
                                                        uint16_t* dst, long long dst_stride,
                                                        long long tokens, int per_token,
                                                        const int* __restrict__ pos,
                                                        double log2_theta) {
  __shared__ float s_cos[kRopeDim / 2], s_sin[kRopeDim / 2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (long long t = blockIdx.x; t < tokens; t += gridDim.x) {
    if (warp == 0) rope_angle(lane, pos[t], log2_theta, &s_cos[lane], &s_sin[lane]);
    __syncthreads();
    const float c = s_cos[lane], sn = s_sin[lane];
    const int j0 = int(blockIdx.y) * 64 + warp * 8;
    uint32_t in[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (j0 + u < per_token)
        in[u] = *reinterpret_cast<const uint32_t*>(
            src + (t * per_token + j0 + u) * src_stride + 2 * lane);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (j0 + u < per_token) {
        const float x0 = bf16_to_f32(uint16_t(in[u] & 0xFFFF));
        const float x1 = bf16_to_f32(uint16_t(in[u] >> 16));
        const float y0 = x0 * c - x1 * sn, y1 = x0 * sn + x1 * c;
        *reinterpret_cast<uint32_t*>(dst + (t * per_token + j0 + u) * dst_stride + 2 * lane) =
            uint32_t(f32_to_bf16(y0)) | (uint32_t(f32_to_bf16(y1)) << 16);
      }
    }
    __syncthreads();  // s_cos / s_sin are reused by the next token
  }
}

// ------------------------------------------------------------------------------ host
struct Layout {
  uint64_t cq, qf, kvf, scratch, total;  // byte offsets into the workspace, and its size
};

uint64_t round256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

Layout layout_of(const TqPrologueSpec& s) {
  const uint64_t T = s.x.shape[0], rq = s.w_qa.shape[0], H = uint64_t(s.heads);
  const uint64_t dn = uint64_t(s.nope_dim), dr = uint64_t(s.rope_dim);
  Layout l;
  l.cq = 0;
  l.qf = l.cq + round256(T * rq * 2);
  l.kvf = l.qf + round256(T * H * (dn + dr) * 2);
  l.scratch = l.kvf + round256(T * (kLatent + dr) * 2);
  l.total = l.scratch + kCublasScratch;
  return l;
}

// Decode-sized batches (T <= 128 tokens) take the weight-streaming projections of tq_proj.cu
// for the narrow projections (q_a, kv_a: at most one 128-row weight tile per two SMs, so K is
// split over a cluster); wide ones (q_b) stay with the library GEMM, which streams them faster.
bool use_proj(const TqPrologueSpec& s) {
  return s.x.shape[0] >= 1 && s.x.shape[0] <= uint64_t(kProjMaxTokens) &&
         s.x.shape[1] >= 128 && s.w_qa.shape[0] >= 128;
}

bool narrow(int n, int sms) { return 2 * ((n + 127) / 128) <= sms; }

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

// Per device: a non-blocking side stream and the fork / join events of the two branches, created
// on the first call with that device current.
struct Side {
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  cudaEvent_t qf_ready = nullptr;  // q's RoPE starts on the side stream once q_b is written
};

Side* side_for(int device) {
  static std::mutex mu;
  static Side cache[128];
  if (device < 0 || device >= 128) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  Side& sd = cache[device];
  if (!sd.stream) {
    Side made;
    if (cudaStreamCreateWithFlags(&made.stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&made.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&made.join, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&made.qf_ready, cudaEventDisableTiming) != cudaSuccess)
      return nullptr;
    sd = made;
  }
  return &sd;
}

// Row-major C[M, N] = A[M, K] . B[N, K]^T with A, B, C packed: cuBLAS sees the column-major
// C^T = B . A^T (op(B) = T).
cublasStatus_t gemm_nt(const Blas* b, cublasHandle_t h, const void* A, const void* B, void* C,
                       int M, int N, int K) {
  const float one = 1.f, zero = 0.f;
  return b->gemm(h, CUBLAS_OP_T, CUBLAS_OP_N, N, M, K, &one, B, CUDA_R_16BF, K, A, CUDA_R_16BF, K,
                 &zero, C, CUDA_R_16BF, N, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
}

std::mutex& blas_mutex() {
  static std::mutex mu;
  return mu;
}

}  // namespace prologue
}  // namespace tq

extern "C" int32_t tq_mla_prologue_workspace_bytes(const TqPrologueSpec* spec, uint64_t* bytes) {
  TqContractError e{nullptr, TQ_OK};
  const int32_t st = tq::prologue_validate(spec, &e);
  if (st != TQ_OK) return st;
  if (!bytes) return TQ_ERR_INVALID_ARGUMENT;
  *bytes = tq::prologue::layout_of(*spec).total;
  return TQ_OK;
}

extern "C" int32_t tq_mla_prologue(const TqPrologueSpec* spec, void* workspace,
                                   uint64_t workspace_bytes, int32_t* device_flags, void* stream,
                                   TqContractError* err) {
  using namespace tq::prologue;
  auto fail = [&](const char* field, int32_t kind) {
    if (err) { err->field = field; err->kind = kind; }
    return kind;
  };
  const int32_t st = tq::prologue_validate(spec, err);
  if (st != TQ_OK) return st;
  const TqPrologueSpec& s = *spec;
  const Layout l = layout_of(s);
  const uint64_t T64 = s.x.shape[0];
  if (T64 == 0) return fail(nullptr, TQ_OK);
  if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 || workspace_bytes < l.total)
    return fail("workspace", TQ_ERR_WORKSPACE);
  const Blas* b = blas();
  if (!b) return fail("libcublas", TQ_ERR_UNSUPPORTED);
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return fail("device", TQ_ERR_CUDA);
  const int sms = sm_count(device);
  if (sms <= 0) return fail("device", TQ_ERR_CUDA);
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);

  const int T = int(T64), dm = int(s.x.shape[1]), rq = int(s.w_qa.shape[0]), H = s.heads;
  const int dn = s.nope_dim, dr = s.rope_dim, width = kLatent + dr;
  char* ws = static_cast<char*>(workspace);
  uint16_t* cq = reinterpret_cast<uint16_t*>(ws + l.cq);
  uint16_t* qf = reinterpret_cast<uint16_t*>(ws + l.qf);
  uint16_t* kvf = reinterpret_cast<uint16_t*>(ws + l.kvf);
  const void* x = reinterpret_cast<const void*>(s.x.device_address);
  uint16_t* q = reinterpret_cast<uint16_t*>(s.q.device_address);
  const int* pos = reinterpret_cast<const int*>(s.pos.device_address);
  const double log2_theta = std::log2(double(s.rope_theta));
  const long long cap = 8ll * sms;
  Side* sd = side_for(device);
  if (!sd) return fail("side_stream", TQ_ERR_CUDA);
  // The cache half of the step, fed to the writer: kvf viewed as bf16 [T, W] rows.
  TqKvWriteSpec w;
  std::memset(&w, 0, sizeof(w));
  w.src.shape[0] = T64;
  w.src.shape[1] = uint64_t(width);
  w.src.strides_bytes[0] = uint64_t(width) * 2;
  w.src.strides_bytes[1] = 2;
  w.src.rank = 2;
  w.src.dtype = TQ_DTYPE_BF16;
  w.src.device_address = reinterpret_cast<uint64_t>(kvf);
  w.src.buffer_bytes = T64 * uint64_t(width) * 2;
  w.kv = s.kv;
  w.page_table = s.page_table;
  w.seq_id = s.seq_id;
  w.pos = s.pos;
  w.kv_format = s.kv_format;
  w.norm_weight = s.kv_norm;
  w.norm_eps = s.kv_eps;
  {
    std::lock_guard<std::mutex> lock(blas_mutex());
    cublasHandle_t h = handle_for(device);
    if (!h) return fail("cublas_handle", TQ_ERR_CUDA);
    // Fork: the cache branch (steps 6-7) runs on this device's side stream beside the query
    // branch (steps 1-5) on the caller's stream; each branch has its own half of the cuBLAS
    // scratch. Both are joined back into the caller's stream before returning, also on errors.
    if (cudaEventRecord(sd->fork, cs) != cudaSuccess ||
        cudaStreamWaitEvent(sd->stream, sd->fork, 0) != cudaSuccess)
      return fail("fork", TQ_ERR_CUDA);
    const char* bad = nullptr;
    int32_t status = TQ_OK;
    constexpr uint64_t kHalf = kCublasScratch / 2;
    const bool proj = use_proj(s);
    // Decode sizes: the weight-streaming projections, K splits balanced for this device.
    auto project = [&](const void* in, uint64_t wt, uint16_t* out, int k, int n,
                       cudaStream_t st) {
      tq::ProjLaunch P;
      P.x = static_cast<const uint16_t*>(in);
      P.w = reinterpret_cast<const uint16_t*>(wt);
      P.t = T;
      P.k = k;
      P.n = n;
      P.splits = tq::proj_splits(n, k, T, sms);
      P.out = out;
      P.flags = device_flags;
      return tq::proj_launch(P, st) == TQ_OK;
    };
    // 6: kvf = x . w_kva^T, its RoPE slice rotated in place; 7: norm and paged write.
    if (proj && narrow(width, sms)) {
      if (!project(x, s.w_kva.device_address, kvf, dm, width, sd->stream)) bad = "proj_kv_a";
    } else if (b->set_stream(h, sd->stream) != CUBLAS_STATUS_SUCCESS ||
               b->set_workspace(h, ws + l.scratch + kHalf, kHalf) != CUBLAS_STATUS_SUCCESS) {
      bad = "cublas_setup";
    } else if (gemm_nt(b, h, x, reinterpret_cast<const void*>(s.w_kva.device_address), kvf, T,
                       width, dm) != CUBLAS_STATUS_SUCCESS) {
      bad = "gemm_kv_a";
    }
    if (!bad && dr) {
      rope_rows_kernel<<<int(T < cap ? T : cap), 256, 0, sd->stream>>>(
          kvf + kLatent, width, kvf + kLatent, width, T, 1, pos, log2_theta);
      if (cudaGetLastError() != cudaSuccess) bad = "launch";
    }
    if (!bad) {
      status = tq_kv_write(&w, device_flags, sd->stream, err);
      if (status != TQ_OK) bad = "kv_write";
    }
    // 1-2: cq = rms(x . w_qa^T) * q_norm; 3: qf = cq . w_qb^T
    if (!bad && (b->set_stream(h, cs) != CUBLAS_STATUS_SUCCESS ||
                 b->set_workspace(h, ws + l.scratch, kHalf) != CUBLAS_STATUS_SUCCESS))
      bad = "cublas_setup";
    if (!bad && (proj && narrow(rq, sms) ? !project(x, s.w_qa.device_address, cq, dm, rq, cs)
                      : gemm_nt(b, h, x, reinterpret_cast<const void*>(s.w_qa.device_address), cq,
                                T, rq, dm) != CUBLAS_STATUS_SUCCESS))
      bad = "gemm_q_a";
    if (!bad) {
      rms_rows_kernel<<<int(T < cap ? T : cap), 256, 0, cs>>>(
          cq, rq, T, reinterpret_cast<const uint16_t*>(s.q_norm.device_address), s.q_eps);
      if (proj && narrow(H * (dn + dr), sms)
              ? !project(cq, s.w_qb.device_address, qf, rq, H * (dn + dr), cs)
               : gemm_nt(b, h, cq, reinterpret_cast<const void*>(s.w_qb.device_address), qf, T,
                         H * (dn + dr), rq) != CUBLAS_STATUS_SUCCESS)
        bad = "gemm_q_b";
    }
    // 5: the RoPE slices of q, which need only qf: on the side stream (its cache branch is
    // queued ahead), beside the absorption, which writes the other columns of q's rows.
    if (!bad && dr) {
      if (cudaEventRecord(sd->qf_ready, cs) != cudaSuccess ||
          cudaStreamWaitEvent(sd->stream, sd->qf_ready, 0) != cudaSuccess) {
        bad = "fork";
      } else {
        rope_rows_kernel<<<dim3(unsigned(T < cap ? T : cap), unsigned((H + 63) / 64)), 256, 0,
                           sd->stream>>>(qf + dn, dn + dr, q + kLatent, width, T, H, pos,
                                         log2_theta);
        if (cudaGetLastError() != cudaSuccess) bad = "launch";
      }
    }
    // 4: per head h, row-major q[:, h, :512] = qf[:, h, :Dn] . w_uk[h]; column-major that is
    // q^T = w_uk[h]^T . qf^T with w_uk[h] seen as a 512 x Dn matrix (ld 512), qf[:, h] as
    // Dn x T (ld H (Dn + Dr)) and q[:, h] as 512 x T (ld H W).
    const float one = 1.f, zero = 0.f;
    if (!bad && b->gemm_batched(h, CUBLAS_OP_N, CUBLAS_OP_N, kLatent, T, dn, &one,
                                reinterpret_cast<const void*>(s.w_uk.device_address), CUDA_R_16BF,
                                kLatent, (long long)dn * kLatent, qf, CUDA_R_16BF, H * (dn + dr),
                                dn + dr, &zero, q, CUDA_R_16BF, H * width, width, H,
                                CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT) != CUBLAS_STATUS_SUCCESS)
      bad = "gemm_absorb";
    if (!bad && cudaGetLastError() != cudaSuccess) bad = "launch";
    // Join.
    if (cudaEventRecord(sd->join, sd->stream) != cudaSuccess ||
        cudaStreamWaitEvent(cs, sd->join, 0) != cudaSuccess)
      return fail("join", TQ_ERR_CUDA);
    if (bad) return status != TQ_OK ? status : fail(bad, TQ_ERR_CUDA);
  }
  return fail(nullptr, TQ_OK);
}
