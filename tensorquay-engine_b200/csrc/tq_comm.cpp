// Communicator of one rank (one GPU worker) and the cross-device merge of a context split.
//
// The reference plans one NCCL communicator per GPU worker behind a `Comm` trait
// (docs/ARCHITECTURE.md:136-137) and, as a later option, decode context parallelism: every GPU
// holds part of each long sequence's pages (docs/ARCHITECTURE.md:240-241,313). Its lifecycle
// rules (docs/ARCHITECTURE.md:242-254) are kept: a communicator whose collective failed is
// aborted and never reused.
//
// NCCL is opened at run time (dlopen of libnccl.so.2). In a process that already has an NCCL
// loaded (PyTorch brings its own) the loader returns that same library, so there is one NCCL
// per process; elsewhere the system's is used. Only the types come from nccl.h.
//
// tq_mla_context_merge = one grouped NCCL all-gather of the f32 partial outputs and their lse
// into caller-owned receive buffers on the caller's stream, then tq_mla_combine (the LSE merge
// kernel) over the G gathered parts.
//
// tq_peer_merge_* = the same merge without a collective on the step: every rank's partials live
// in an exchange region exported with CUDA IPC; the handles are all-gathered once over NCCL at
// creation, and each step one kernel per rank reads its peers' partials over NVLink
// (tq_peer_merge.cu). Plain peer loads and stores only: no multicast of any kind.

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <new>

#include "tq_contracts.h"

namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*);
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*comm_destroy)(ncclComm_t);
  ncclResult_t (*comm_abort)(ncclComm_t);
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t);
  ncclResult_t (*group_start)();
  ncclResult_t (*group_end)();
  bool ok = false;
};

const NcclApi* nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    auto sym = [&](const char* name) { return dlsym(h, name); };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
    api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(sym("ncclCommAbort"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
    api.group_start = reinterpret_cast<decltype(api.group_start)>(sym("ncclGroupStart"));
    api.group_end = reinterpret_cast<decltype(api.group_end)>(sym("ncclGroupEnd"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.comm_abort &&
             api.all_gather && api.group_start && api.group_end;
  });
  return api.ok ? &api : nullptr;
}

static_assert(sizeof(TqCommId) == sizeof(ncclUniqueId), "communicator id size");

}  // namespace

struct TqComm {
  ncclComm_t comm;
  int32_t nranks;
  int32_t rank;
  int32_t device;
  int32_t failed;  // a collective failed: only abort/destroy remain
};

struct TqPeerMerge {
  TqComm* comm;
  int32_t nranks, rank, device;
  uint64_t tokens, heads, bytes;
  uint8_t* own;                             // this rank's exchange region (cudaMalloc)
  uint8_t* mapped[tq::kPeerMaxRanks];       // every rank's region as mapped on this device
};

namespace {

// A small all-gather over `comm` on a private stream, waited for: `bytes` from this rank, the
// ranks' contributions in rank order in `host_out`.
int32_t gather_bytes(TqComm* comm, const void* mine, uint64_t bytes, void* host_out) {
  const NcclApi* api = nccl();
  if (!api || comm->failed) return TQ_ERR_COMM;
  uint8_t* d = nullptr;
  cudaStream_t st = nullptr;
  int32_t rc = TQ_OK;
  if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) return TQ_ERR_CUDA;
  if (cudaMalloc(&d, bytes * uint64_t(comm->nranks)) != cudaSuccess) {
    cudaStreamDestroy(st);
    return TQ_ERR_CUDA;
  }
  if (cudaMemcpyAsync(d + bytes * uint64_t(comm->rank), mine, bytes, cudaMemcpyHostToDevice,
                      st) != cudaSuccess)
    rc = TQ_ERR_CUDA;
  if (rc == TQ_OK && api->all_gather(d + bytes * uint64_t(comm->rank), d, size_t(bytes), ncclInt8,
                                     comm->comm, st) != ncclSuccess) {
    comm->failed = 1;
    rc = TQ_ERR_COMM;
  }
  if (rc == TQ_OK && (cudaMemcpyAsync(host_out, d, bytes * uint64_t(comm->nranks),
                                      cudaMemcpyDeviceToHost, st) != cudaSuccess ||
                      cudaStreamSynchronize(st) != cudaSuccess))
    rc = TQ_ERR_CUDA;
  cudaFree(d);
  cudaStreamDestroy(st);
  return rc;
}

}  // namespace

extern "C" {

int32_t tq_comm_unique_id(TqCommId* id) {
  if (!id) return TQ_ERR_INVALID_ARGUMENT;
  const NcclApi* api = nccl();
  if (!api) return TQ_ERR_COMM;
  ncclUniqueId u;
  if (api->get_unique_id(&u) != ncclSuccess) return TQ_ERR_COMM;
  std::memcpy(id, &u, sizeof(u));
  return TQ_OK;
}

int32_t tq_comm_init(const TqCommId* id, int32_t nranks, int32_t rank, TqComm** comm) {
  if (!id || !comm || nranks < 1 || rank < 0 || rank >= nranks) return TQ_ERR_INVALID_ARGUMENT;
  *comm = nullptr;
  const NcclApi* api = nccl();
  if (!api) return TQ_ERR_COMM;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return TQ_ERR_CUDA;
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  ncclComm_t c = nullptr;
  if (api->comm_init_rank(&c, nranks, u, rank) != ncclSuccess) {
    if (c) api->comm_abort(c);
    return TQ_ERR_COMM;
  }
  TqComm* t = new (std::nothrow) TqComm{c, nranks, rank, device, 0};
  if (!t) {
    api->comm_abort(c);
    return TQ_ERR_INVALID_ARGUMENT;
  }
  *comm = t;
  return TQ_OK;
}

int32_t tq_comm_abort(TqComm* comm) {
  if (!comm) return TQ_ERR_INVALID_ARGUMENT;
  const NcclApi* api = nccl();
  const int32_t st = (api && api->comm_abort(comm->comm) == ncclSuccess) ? TQ_OK : TQ_ERR_COMM;
  delete comm;
  return st;
}

int32_t tq_comm_destroy(TqComm* comm) {
  if (!comm) return TQ_ERR_INVALID_ARGUMENT;
  if (comm->failed) return tq_comm_abort(comm);
  const NcclApi* api = nccl();
  const int32_t st = (api && api->comm_destroy(comm->comm) == ncclSuccess) ? TQ_OK : TQ_ERR_COMM;
  delete comm;
  return st;
}

int32_t tq_comm_rank(const TqComm* comm, int32_t* rank, int32_t* nranks) {
  if (!comm || !rank || !nranks) return TQ_ERR_INVALID_ARGUMENT;
  *rank = comm->rank;
  *nranks = comm->nranks;
  return TQ_OK;
}

int32_t tq_mla_context_merge(const TqContextMergeParams* p, TqComm* comm, void* stream) {
  if (!p || !comm) return TQ_ERR_INVALID_ARGUMENT;
  if (comm->failed) return TQ_ERR_COMM;
  if (p->tokens == 0 || p->heads == 0) return TQ_OK;
  if (!p->part_out || !p->part_lse || !p->gather_out || !p->gather_lse || !p->out || !p->lse)
    return TQ_ERR_INVALID_ARGUMENT;
  if (p->out_dtype != TQ_DTYPE_BF16 && p->out_dtype != TQ_DTYPE_F32)
    return TQ_ERR_INVALID_ARGUMENT;
  if ((p->part_out | p->gather_out | p->out | p->out_stride_token | p->out_stride_head) % 16 ||
      (p->part_lse | p->gather_lse | p->lse) % 4)
    return TQ_ALIGNMENT;
  const uint64_t rows = p->tokens * p->heads;
  if (p->heads > (uint64_t(1) << 31) || rows / p->heads != p->tokens || rows > (uint64_t(1) << 40))
    return TQ_ERR_INVALID_ARGUMENT;
  const uint64_t g = uint64_t(comm->nranks);
  if (p->gather_out_bytes < g * rows * 512 * 4 || p->gather_lse_bytes < g * rows * 4)
    return TQ_CAPACITY;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return TQ_ERR_CUDA;
  if (device != comm->device) return TQ_ERR_INVALID_ARGUMENT;
  const NcclApi* api = nccl();
  if (!api) return TQ_ERR_COMM;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  bool ok = api->group_start() == ncclSuccess;
  if (ok) {
    ok = api->all_gather(reinterpret_cast<const void*>(p->part_out),
                         reinterpret_cast<void*>(p->gather_out), size_t(rows * 512), ncclFloat32,
                         comm->comm, st) == ncclSuccess;
    ok = api->all_gather(reinterpret_cast<const void*>(p->part_lse),
                         reinterpret_cast<void*>(p->gather_lse), size_t(rows), ncclFloat32,
                         comm->comm, st) == ncclSuccess && ok;
    ok = api->group_end() == ncclSuccess && ok;
  }
  if (!ok) {
    comm->failed = 1;
    return TQ_ERR_COMM;
  }
  TqCombineParams cp;
  std::memset(&cp, 0, sizeof(cp));
  cp.parts = g;
  cp.tokens = p->tokens;
  cp.heads = p->heads;
  cp.part_out = p->gather_out;
  cp.part_lse = p->gather_lse;
  cp.out = p->out;
  cp.lse = p->lse;
  cp.out_stride_token = p->out_stride_token;
  cp.out_stride_head = p->out_stride_head;
  cp.out_dtype = p->out_dtype;
  return tq_mla_combine(&cp, stream);
}

int32_t tq_peer_merge_create(TqComm* comm, uint64_t tokens, uint64_t heads, TqPeerMerge** out) {
  if (!comm || !out) return TQ_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  if (comm->failed) return TQ_ERR_COMM;
  if (comm->nranks < 1 || comm->nranks > tq::kPeerMaxRanks) return TQ_ERR_UNSUPPORTED;
  const uint64_t rows = tokens * heads;
  if (tokens == 0 || heads == 0 || heads > (uint64_t(1) << 31) || rows / heads != tokens ||
      rows > (uint64_t(1) << 32))
    return TQ_ERR_INVALID_ARGUMENT;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return TQ_ERR_CUDA;
  if (device != comm->device) return TQ_ERR_INVALID_ARGUMENT;
  TqPeerMerge* pm = new (std::nothrow) TqPeerMerge;
  if (!pm) return TQ_ERR_INVALID_ARGUMENT;
  std::memset(pm, 0, sizeof(*pm));
  pm->comm = comm;
  pm->nranks = comm->nranks;
  pm->rank = comm->rank;
  pm->device = device;
  pm->tokens = tokens;
  pm->heads = heads;
  pm->bytes = (tq::kPeerHeaderBytes + rows * 2048 + rows * 4 + 255) & ~uint64_t(255);
  if (cudaMalloc(&pm->own, pm->bytes) != cudaSuccess) {
    delete pm;
    return TQ_ERR_CUDA;
  }
  // The header is zero before any peer can learn the region exists.
  if (cudaMemset(pm->own, 0, tq::kPeerHeaderBytes) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(pm->own);
    delete pm;
    return TQ_ERR_CUDA;
  }
  pm->mapped[pm->rank] = pm->own;
  cudaIpcMemHandle_t mine;
  cudaIpcMemHandle_t all[tq::kPeerMaxRanks];
  int32_t rc = TQ_OK;
  if (pm->nranks > 1) {
    if (cudaIpcGetMemHandle(&mine, pm->own) != cudaSuccess) rc = TQ_ERR_CUDA;
    if (rc == TQ_OK) rc = gather_bytes(comm, &mine, sizeof(mine), all);
    for (int r = 0; rc == TQ_OK && r < pm->nranks; ++r) {
      if (r == pm->rank) continue;
      void* p = nullptr;
      if (cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
        rc = TQ_ERR_CUDA;
      else
        pm->mapped[r] = static_cast<uint8_t*>(p);
    }
  }
  if (rc != TQ_OK) {
    for (int r = 0; r < pm->nranks; ++r)
      if (r != pm->rank && pm->mapped[r]) cudaIpcCloseMemHandle(pm->mapped[r]);
    cudaFree(pm->own);
    delete pm;
    return rc;
  }
  *out = pm;
  return TQ_OK;
}

int32_t tq_peer_merge_partials(const TqPeerMerge* pm, uint64_t* part_out, uint64_t* part_lse) {
  if (!pm || !part_out || !part_lse) return TQ_ERR_INVALID_ARGUMENT;
  const uint64_t rows = pm->tokens * pm->heads;
  *part_out = reinterpret_cast<uint64_t>(pm->own) + tq::kPeerHeaderBytes;
  *part_lse = *part_out + rows * 2048;
  return TQ_OK;
}

int32_t tq_peer_merge(TqPeerMerge* pm, uint64_t out, uint64_t lse, uint64_t out_stride_token,
                      uint64_t out_stride_head, int32_t out_dtype, void* stream) {
  if (!pm || !out || !lse) return TQ_ERR_INVALID_ARGUMENT;
  if (out_dtype != TQ_DTYPE_BF16 && out_dtype != TQ_DTYPE_F32) return TQ_ERR_INVALID_ARGUMENT;
  if ((out | out_stride_token | out_stride_head) % 16 || lse % 4) return TQ_ALIGNMENT;
  if (out_stride_head < (out_dtype == TQ_DTYPE_F32 ? 2048u : 1024u) ||
      out_stride_token < out_stride_head * pm->heads)
    return TQ_STRIDE;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return TQ_ERR_CUDA;
  if (device != pm->device) return TQ_ERR_INVALID_ARGUMENT;
  tq::PeerMergeLaunch L;
  std::memset(&L, 0, sizeof(L));
  for (int r = 0; r < pm->nranks; ++r) L.regions[r] = pm->mapped[r];
  L.nranks = pm->nranks;
  L.rank = pm->rank;
  L.tokens = pm->tokens;
  L.heads = pm->heads;
  L.out = reinterpret_cast<uint8_t*>(out);
  L.lse = reinterpret_cast<float*>(lse);
  L.out_stride_token = out_stride_token;
  L.out_stride_head = out_stride_head;
  L.out_bf16 = out_dtype == TQ_DTYPE_BF16;
  return tq::peer_merge_launch(L, stream);
}

int32_t tq_peer_merge_read_error(const TqPeerMerge* pm, void* stream, int32_t* flags) {
  if (!pm || !flags) return TQ_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t v = 0;
  if (cudaMemcpyAsync(&v, pm->own + 4 * tq::kPeerHdrError, sizeof(v), cudaMemcpyDeviceToHost,
                      st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return TQ_ERR_CUDA;
  *flags = v;
  return TQ_OK;
}

int32_t tq_peer_merge_destroy(TqPeerMerge* pm) {
  if (!pm) return TQ_ERR_INVALID_ARGUMENT;
  int32_t rc = TQ_OK;
  if (cudaDeviceSynchronize() != cudaSuccess) rc = TQ_ERR_CUDA;
  uint8_t token = 0, tokens[tq::kPeerMaxRanks];
  // Every rank has stopped touching the others' regions before any mapping goes away, and every
  // mapping of a region is closed before its owner frees it.
  if (pm->nranks > 1 && !pm->comm->failed) {
    if (gather_bytes(pm->comm, &token, 1, tokens) != TQ_OK) rc = TQ_ERR_COMM;
  }
  for (int r = 0; r < pm->nranks; ++r)
    if (r != pm->rank && pm->mapped[r] && cudaIpcCloseMemHandle(pm->mapped[r]) != cudaSuccess)
      rc = TQ_ERR_CUDA;
  if (pm->nranks > 1 && !pm->comm->failed) {
    if (gather_bytes(pm->comm, &token, 1, tokens) != TQ_OK) rc = TQ_ERR_COMM;
  }
  if (cudaFree(pm->own) != cudaSuccess) rc = TQ_ERR_CUDA;
  delete pm;
  return rc;
}

}  // extern "C"
