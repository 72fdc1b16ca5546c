/*
 * tq_mla.h - C ABI of the B200 (sm_100a) absorbed-MLA paged-attention library (libtq_mla.so).
 *
 * Plain C types only: numeric device addresses, byte sizes, status codes. No exceptions cross
 * this boundary and the library allocates no device memory on the launch path: the caller owns
 * every buffer, including the workspace whose size tq_mla_workspace_bytes reports.
 *
 * Reference interfaces each entry point replaces (paths inside TensorQuay/tensorquay-engine):
 *   tq_mla_validate          SmlaParams::new            crates/tq-core/src/contracts.rs:437-493
 *   tq_mla_prefill_validate  the SMLA-PF contract       docs/TEST-PLAN.md:195,410-413 (planned)
 *   tq_mla_should_launch     SmlaParams::should_launch  crates/tq-core/src/contracts.rs:509-511
 *   tq_mla_decode            sparse_mla_decode launcher docs/ARCHITECTURE.md:111-113 (planned),
 *                            dense paged form; numerics reference/src/tq_reference/
 *                            mla_attention.py:135-169
 *   tq_mla_prefill           SMLA-PF launcher           docs/TEST-PLAN.md:410-413 (planned)
 *   tq_mla_combine           split-K merge              docs/TEST-PLAN.md:206-207,220,247
 *   tq_comm_*                the planned NCCL Comm      docs/ARCHITECTURE.md:136-137, lifecycle
 *                            (per GPU worker)           :242-254 (abort, never reuse a failed one)
 *   tq_mla_context_merge     decode context parallelism docs/ARCHITECTURE.md:240-241,313 (planned
 *                            "later option"): all-gather of per-device partials + LSE merge
 *   tq_philox_words          tq_testkit::philox::fill_words crates/tq-testkit/src/philox.rs:78-98
 *   tq_philox_block          tq_testkit::philox::block      crates/tq-testkit/src/philox.rs:57-70
 *   tq_philox_uniform_f32    tq_testkit::philox::uniform_f32 crates/tq-testkit/src/philox.rs:109-111
 */
#ifndef TQ_MLA_H
#define TQ_MLA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Storage element types (contracts.rs:41-50). */
enum { TQ_DTYPE_BF16 = 0, TQ_DTYPE_I32 = 1, TQ_DTYPE_F32 = 2, TQ_DTYPE_U8 = 3 };

/* Paged row formats (contracts.rs:129-144), plus the 576-wide DeepSeek-style row. */
enum {
  TQ_KV_BF16 = 0,         /* 512 bf16 latent values, 1024 B, q width 512, scale 0.0625   */
  TQ_KV_FP8_E4M3 = 1,     /* 512 E4M3 codes + 4 f32 scales, 528 B; q 512 wide (bf16) */
  TQ_KV_BF16_ROPE576 = 2  /* 512 latent + 64 RoPE bf16, 1152 B, q width 576, any scale > 0  */
};

/* Status codes. 1..12 are the contract violations (contracts.rs:65-90) in declaration order. */
enum {
  TQ_OK = 0,
  TQ_SHAPE = 1, TQ_DTYPE = 2, TQ_DIMENSION = 3, TQ_STRIDE = 4, TQ_ALIGNMENT = 5,
  TQ_ADDRESS = 6, TQ_CAPACITY = 7, TQ_OVERFLOW = 8, TQ_QUERY_COUNT = 9, TQ_SCALE = 10,
  TQ_GROUP = 11, TQ_ALIAS = 12,
  TQ_ERR_INVALID_ARGUMENT = 100, /* null pointer or malformed argument                   */
  TQ_ERR_UNSUPPORTED = 101,      /* validated layout that no kernel here launches        */
  TQ_ERR_WORKSPACE = 102,        /* workspace missing, misaligned or too small           */
  TQ_ERR_CUDA = 103,             /* a CUDA runtime/driver call failed                    */
  TQ_ERR_PARAMS = 104,           /* params not produced by a validate call, or altered   */
  TQ_ERR_RANGE = 105,            /* Philox word range exceeds u64 (philox.md:69-75)      */
  TQ_ERR_COMM = 106              /* NCCL missing, or a collective failed: the communicator
                                    is unusable from then on; abort it and make a new one  */
};

/* Device error flag bits, read back with tq_mla_read_device_error. */
enum {
  TQ_DEV_WAIT_TIMEOUT = 1,  /* a bounded wait gave up; the kernel aborted cleanly          */
  TQ_DEV_PAGE_RANGE = 2,    /* a page-table entry outside [0, pages); the tile read zeros */
  TQ_DEV_SEQ_RANGE = 4,     /* a seq_id outside [0, sequences); the token was left empty  */
  TQ_DEV_TABLE_SHORT = 8,   /* kv_len beyond 64 * page-table width; clamped              */
  TQ_DEV_WORK_OVERFLOW = 16 /* total page work does not fit 31 bits; nothing computed     */
};

/* One tensor declaration (contracts.rs:109-125). rank <= 3; unused trailing axes ignored. */
typedef struct {
  uint64_t shape[3];
  uint64_t strides_bytes[3];
  int32_t rank;
  int32_t dtype;
  uint64_t device_address;
  uint64_t buffer_bytes;
} TqTensorSpec;

/* Dense paged MLA launch metadata (the dense form of SmlaSpec, contracts.rs:182-209).
 *   q          bf16 [T, H, Dqk]   Dqk = 512 (TQ_KV_BF16) or 576 (TQ_KV_BF16_ROPE576)
 *   kv         u8   [P, 64, payload] with strides [64 r, r, 1], r >= payload, r % 16 == 0
 *   page_table i32  [S, L]
 *   seq_id     i32  [T]      q_pos i32 [T]      kv_len i32 [S]
 *   out        bf16 or f32 [T, H, 512]          lse   f32 [T, H] (natural log)
 * Token t attends to positions [0, min(kv_len[seq_id[t]], q_pos[t] + 1)) of its sequence. */
typedef struct {
  TqTensorSpec q, kv, page_table, seq_id, q_pos, kv_len, out, lse;
  int32_t kv_format;
  float softmax_scale;
} TqMlaSpec;

/* A rejected contract: stable field name (static storage) and violation kind. */
typedef struct {
  const char* field;
  int32_t kind;
} TqContractError;

/* Validated parameters. Produced only by the validate calls; launches re-check the digest. */
typedef struct {
  TqMlaSpec spec;
  uint64_t tokens, heads, sequences, slots, pages, qk_width, row_stride;
  int32_t max_queries_per_sequence; /* 4 for decode plans, 0 for prefill plans */
  int32_t should_launch;            /* tokens != 0                              */
  TqTensorSpec idx;                 /* sparse plans: i32 [T, K]; zeros otherwise */
  TqTensorSpec k_len;               /* sparse plans: i32 [T]; zeros otherwise    */
  uint64_t topk;                    /* K of a sparse plan, 0 otherwise            */
  int32_t sparse;                   /* 1 for a sparse plan (tq_mla_sparse_validate) */
  int32_t reserved;
  uint64_t digest;
} TqMlaParams;

/* Merge of G partial results (fp32 outputs normalised per part, natural-log lse):
 *   part_out f32 [G, T, H, 512] packed, part_lse f32 [G, T, H] packed,
 *   out bf16 or f32 [T, H, 512] (padded outer strides allowed), lse f32 [T, H] packed. */
typedef struct {
  uint64_t parts, tokens, heads;
  uint64_t part_out, part_lse; /* device addresses */
  uint64_t out, lse;
  uint64_t out_stride_token, out_stride_head; /* bytes */
  int32_t out_dtype;
} TqCombineParams;

/* Byte offsets of the scheduler metadata inside a workspace (for inspection and tests). */
typedef struct {
  uint64_t total_bytes;
  uint64_t header;        /* int32[16]: error, virtual pages, quota, n_combine, n_empty, pairs*/
  uint64_t unit_n;        /* int32[T]  visible keys per token                               */
  uint64_t unit_pages;    /* int32[T]                                                       */
  uint64_t unit_gstart;   /* int32[T]  virtual position of the first page                   */
  uint64_t unit_first;    /* int32[T]  first CTA pair touching the token (-1 if none)       */
  uint64_t unit_nsplit;   /* int32[T]                                                       */
  uint64_t unit_split_off;/* int32[T]                                                       */
  uint64_t pair_begin;    /* int32[pairs] first token of each CTA pair (-1 if idle)          */
  uint64_t combine_list;  /* int32[T]                                                       */
  uint64_t empty_list;    /* int32[T]                                                       */
  uint64_t part_lse;      /* f32[2*pairs, 128]                                              */
  uint64_t part_out;      /* f32[2*pairs, 128 column quads, 128 rows, 4]                    */
  uint64_t sparse_rows;   /* int32[T, K] sparse plans: each token's valid pool rows, in order */
  uint64_t sparse_count;  /* int32[T]    sparse plans: valid entries per token               */
  int32_t pairs;          /* CTA pairs of the main kernel on this device                    */
} TqWorkspaceLayout;

/* Decode plan: query_counts[n] with n == S, each <= 4, sum == T (contracts.rs:477-490). */
int32_t tq_mla_validate(const TqMlaSpec* spec, const uint8_t* query_counts, uint64_t n,
                        TqMlaParams* params, TqContractError* err);
/* Prefill plan: query_counts[n] with n == S and sum == T; no per-sequence limit. */
int32_t tq_mla_prefill_validate(const TqMlaSpec* spec, const uint32_t* query_counts, uint64_t n,
                                TqMlaParams* params, TqContractError* err);
int32_t tq_mla_should_launch(const TqMlaParams* params);

/* Sparse top-k decode plan: SmlaParams::new with the DSA index tensors (contracts.rs:437-493,
 * SmlaSpec idx / k_len at :196-200; docs/TEST-PLAN.md:190-199).
 *   idx   i32 [T, K], K <= 2051, padded row stride allowed; -1 marks an empty entry
 *   k_len i32 [T]
 * Entry j of token t is valid iff j < k_len[t] and 0 <= idx[t][j] <= q_pos[t] and
 * idx[t][j] < kv_len[seq_id[t]]; token t attends to exactly the rows of its valid entries (an
 * entry listed twice counts twice). Invalid entries are never read. Rows are 512 wide
 * (TQ_KV_BF16 or TQ_KV_FP8_E4M3). The plan is launched with tq_mla_decode / tq_mla_decode_no_alloc
 * like a dense one; the launch grid does not depend on the indices, so a captured launch replays
 * with new idx, k_len, q_pos and kv_len. A page-table entry outside the pool makes its entry
 * invalid and sets TQ_DEV_PAGE_RANGE. */
#define TQ_MLA_MAX_TOPK 2051
int32_t tq_mla_sparse_validate(const TqMlaSpec* spec, const TqTensorSpec* idx,
                               const TqTensorSpec* k_len, const uint8_t* query_counts, uint64_t n,
                               TqMlaParams* params, TqContractError* err);

/* Workspace size and layout for a validated launch on `device` (0-based CUDA ordinal). */
int32_t tq_mla_workspace_bytes(const TqMlaParams* params, int32_t device, uint64_t* bytes);
int32_t tq_mla_workspace_layout(const TqMlaParams* params, int32_t device,
                                TqWorkspaceLayout* layout);

/* Launch on `stream` (a cudaStream_t; NULL = legacy default stream) of the current device.
 * The workspace must be 256-byte aligned and at least tq_mla_workspace_bytes long; calls that
 * share a workspace must be ordered on one stream. `err` (optional) names the field when a
 * launch-time layout requirement fails (q needs 16-byte aligned address and strides for TMA). */
int32_t tq_mla_decode(const TqMlaParams* params, void* workspace, uint64_t workspace_bytes,
                      void* stream, TqContractError* err);
int32_t tq_mla_prefill(const TqMlaParams* params, void* workspace, uint64_t workspace_bytes,
                       void* stream, TqContractError* err);
int32_t tq_mla_combine(const TqCombineParams* params, void* stream);

/* Communicator of one rank of a multi-GPU job (an NCCL communicator, one per GPU worker; NCCL
 * is loaded at run time as libnccl.so.2, so the library has no link-time NCCL dependency and
 * shares the NCCL already loaded into the process, if any).
 *   tq_comm_unique_id   on one rank; the caller sends the 128 bytes to every rank (host side)
 *   tq_comm_init        on every rank, with its GPU current; collective over all ranks
 *   tq_comm_abort       after a failed or timed-out collective (TQ_ERR_COMM): frees it at once
 *   tq_comm_destroy     normal teardown; destroy CUDA graphs holding its collectives first
 * A communicator that reported TQ_ERR_COMM refuses further collectives (TQ_ERR_COMM). */
typedef struct { char internal[128]; } TqCommId;
typedef struct TqComm TqComm;
int32_t tq_comm_unique_id(TqCommId* id);
int32_t tq_comm_init(const TqCommId* id, int32_t nranks, int32_t rank, TqComm** comm);
int32_t tq_comm_abort(TqComm* comm);
int32_t tq_comm_destroy(TqComm* comm);
int32_t tq_comm_rank(const TqComm* comm, int32_t* rank, int32_t* nranks);

/* Cross-device merge of a context split: each of the G ranks holds the partial result of the
 * same T query tokens over its own page range (f32 out normalised over that range and its
 * natural-log lse, e.g. a tq_mla_decode with f32 out). The partials of all ranks are
 * all-gathered into gather_out f32 [G, T, H, 512] and gather_lse f32 [G, T, H] (caller-owned,
 * packed, at least gather_*_bytes long), then merged by log-sum-exp into out (bf16 or f32
 * [T, H, 512], padded outer strides allowed) and lse f32 [T, H] on every rank, as
 * tq_mla_combine does. part_out and part_lse are packed [T, H, 512] / [T, H]. Every rank makes
 * the same call with the same T and H, in the same order as its other collectives on `comm`.
 * Device addresses and strides must be 16-byte aligned. */
typedef struct {
  uint64_t tokens, heads;
  uint64_t part_out, part_lse;              /* this rank's partials (device)       */
  uint64_t gather_out, gather_lse;          /* receive buffers (device)            */
  uint64_t gather_out_bytes, gather_lse_bytes;
  uint64_t out, lse;                        /* merged result (device)              */
  uint64_t out_stride_token, out_stride_head; /* bytes                             */
  int32_t out_dtype;
} TqContextMergeParams;
int32_t tq_mla_context_merge(const TqContextMergeParams* params, TqComm* comm, void* stream);

/* The same merge over NVLink peer memory, with no collective on the step (the planned "NVLink
 * LSE merge" of decode context parallelism, docs/ARCHITECTURE.md:240-241,313):
 *   tq_peer_merge_create     collective over `comm` (all ranks, same tokens and heads, each with
 *                            its GPU current): allocates this rank's exchange region (a 256-byte
 *                            header, f32 partial out [T, H, 512], f32 lse [T, H]), exports it
 *                            with CUDA IPC and opens every peer's (handles all-gathered once
 *                            over NCCL). Up to 8 ranks.
 *   tq_peer_merge_partials   device addresses of this rank's partials in its region: decode
 *                            into them (tq_mla_decode with f32 out, packed [T, H, 512] and lse)
 *   tq_peer_merge            one kernel on `stream`, after that decode: tells every peer this
 *                            rank's partials are ready, waits for theirs, merges all ranks' rows
 *                            by log-sum-exp reading the peers' partials over NVLink into out
 *                            (bf16 or f32 [T, H, 512], strides in bytes, 16-byte aligned) and lse
 *                            f32 [T, H], then waits until every peer has read this rank's
 *                            partials, so the next decode may overwrite them. Every rank calls it
 *                            once per step, in the same order; the step counter lives on the
 *                            device, so a captured decode + merge replays.
 *   tq_peer_merge_read_error the region's device error flags (synchronises `stream`): a wait
 *                            that gave up after ~2 s (a peer that never arrived) sets
 *                            TQ_DEV_WAIT_TIMEOUT, and every later merge on the plan returns at
 *                            once; destroy it (and the communicator) then.
 *   tq_peer_merge_destroy    collective: waits for the device, closes the peers' mappings and
 *                            frees the region (two small NCCL barriers). */
typedef struct TqPeerMerge TqPeerMerge;
int32_t tq_peer_merge_create(TqComm* comm, uint64_t tokens, uint64_t heads, TqPeerMerge** pm);
int32_t tq_peer_merge_partials(const TqPeerMerge* pm, uint64_t* part_out, uint64_t* part_lse);
int32_t tq_peer_merge(TqPeerMerge* pm, uint64_t out, uint64_t lse, uint64_t out_stride_token,
                      uint64_t out_stride_head, int32_t out_dtype, void* stream);
int32_t tq_peer_merge_read_error(const TqPeerMerge* pm, void* stream, int32_t* flags);
int32_t tq_peer_merge_destroy(TqPeerMerge* pm);

/* Device error flag of the last launch that used `workspace` (synchronises `stream`). */
int32_t tq_mla_read_device_error(const void* workspace, void* stream, int32_t* flags);

/* Decode without any device allocation. No counterpart in the reference: it exists for callers
 * that cannot allocate device memory at launch time, such as an engine that hands all GPU memory
 * to its own pool up front, or code running where cudaMalloc is not allowed.
 * Same plan, inputs, outputs and results as tq_mla_decode, but the workspace is a fixed array
 * inside this library of TQ_MLA_NO_ALLOC_WORKSPACE_BYTES (42 MiB), which every GPU that loads the
 * library keeps until the process exits. A plan whose tq_mla_workspace_bytes exceeds that size
 * returns TQ_ERR_WORKSPACE with field "no_alloc_workspace". On a B200 about 39 MB of the array
 * hold the split partials and the rest 32 bytes per query token, so dense plans fit up to about
 * 160 000 query tokens; a sparse plan also keeps 4 K + 4 bytes per token for its compacted
 * entries, so it fits about 5.1 MB / (4 K + 36) tokens: about 620 at K = 2051. The first call
 * on each device (and the first after that device's context changed) looks up the array's
 * device address, so make it before capturing any stream. All calls share the one array: calls
 * that may overlap on the GPU (other streams, other threads) race and must be serialised by the
 * caller. tq_mla_no_alloc_read_device_error reads the device error flags of the last call on
 * the current device (it synchronises `stream`). */
#define TQ_MLA_NO_ALLOC_WORKSPACE_BYTES (42ull << 20)
int32_t tq_mla_decode_no_alloc(const TqMlaParams* params, void* stream, TqContractError* err);
int32_t tq_mla_no_alloc_read_device_error(void* stream, int32_t* flags);

/* KV cache writer: the planned "latent -> 528 B KV writer" (docs/DEV-PLAN.md:116) over the row
 * formats of docs/HOST-CONTRACTS.md:122-123 and the paged addressing of contracts.rs:182-209.
 *   src        bf16 [T, W]   W = 576 (TQ_KV_BF16_ROPE576) or 512 (TQ_KV_BF16, TQ_KV_FP8_E4M3);
 *                            row stride >= 2 W, address and row stride multiples of 16
 *   kv         u8   [P, 64, payload] with strides [64 r, r, 1], r >= payload, r % 16 == 0
 *   page_table i32  [S, L]    seq_id i32 [T]    pos i32 [T]
 * Row t is written to pool row page_table[seq_id[t]][pos[t] / 64] * 64 + pos[t] % 64: its bf16
 * bits as they are, or, for FP8 rows, 512 E4M3 codes and four f32 tile scales. FP8 rule per
 * 128-value tile: a NaN in the tile gives scale NaN and codes 0x7F; amax == 0 gives scale 0 and
 * codes 0; otherwise scale = amax / 448, inv = 448 / amax and code = E4M3(x * inv), or
 * E4M3(x / scale) when inv overflows (amax below ~1.3e-36); f32 operations rounded to nearest
 * even, E4M3 rounded to nearest even and saturated to +-448. Bytes past the payload are
 * not touched. A row whose seq_id, pos or page entry is out of range is skipped and, when
 * `device_flags` (a device int32, may be null) is given, TQ_DEV_SEQ_RANGE, TQ_DEV_TABLE_SHORT or
 * TQ_DEV_PAGE_RANGE is OR-ed into it. Two rows naming one slot in a call race (either may win).
 * The launch grid depends only on the device and the row count, so a captured call replays
 * for new contents of the same shapes.
 * Optional RMSNorm of each row's 512 latent values before the write (the norm of the planned
 * "kv_a -> norm -> cache write" prologue; docs/DEV-PLAN.md:116): with norm_weight a bf16 [512]
 * tensor (rank 0 switches it off) and norm_eps finite and > 0, each latent value becomes
 * bf16(bf16(x * r) * w) with r = 1 / sqrt(sum(x^2) / 512 + eps): the normalised value rounded to
 * bf16 before the weight multiplies it, the rounding points of the model's RMSNorm
 * (weight * hidden.to(bf16); docs/reviews/2026-09-19-design-review.md:13). All f32 operations
 * are IEEE round-to-nearest (no fused multiply-add); the sum adds each 16-value run in order,
 * then combines the 32 runs pairwise at distances 16, 8, 4, 2, 1. The 64 RoPE values of a 576-wide
 * row are copied unchanged; FP8 rows quantize the normalised bf16 values. */
typedef struct {
  TqTensorSpec src, kv, page_table, seq_id, pos;
  int32_t kv_format;
  TqTensorSpec norm_weight; /* bf16 [512], or rank 0 for no norm */
  float norm_eps;
} TqKvWriteSpec;
int32_t tq_kv_write_validate(const TqKvWriteSpec* spec, TqContractError* err);
int32_t tq_kv_write(const TqKvWriteSpec* spec, int32_t* device_flags, void* stream,
                    TqContractError* err);

/* MLA prologue: the planned "q_a -> norm -> q_b -> absorb; kv_a -> norm -> cache write"
 * (docs/DEV-PLAN.md:116). Two row forms: rope_dim 0, the no-RoPE model of
 * docs/research/glm-5.md:163-167 (q 512 wide; kv_format TQ_KV_BF16 or TQ_KV_FP8_E4M3), and
 * rope_dim 64 with 576-wide rows (kv_format TQ_KV_BF16_ROPE576). With Dr = rope_dim and
 * W = 512 + Dr, for every token t:
 *   cq      = bf16(x[t] . w_qa^T)                                   [Rq]
 *   cqn     = bf16(bf16(rms(cq)) * q_norm)                          [Rq]
 *   qf      = bf16(cqn . w_qb^T)                  per head h:       [Dn | Dr]
 *   q[t, h] = [ bf16(qf[h][:Dn] . w_uk[h]) (the key absorption of mla_attention.py:150)
 *             | bf16(rope(qf[h][Dn:], pos[t])) ]                    [512 | Dr]
 *   kvf     = bf16(x[t] . w_kva^T)                                  [512 | Dr]
 *   row     = [ bf16(bf16(rms(kvf[:512])) * kv_norm) | bf16(rope(kvf[512:], pos[t])) ]
 * and `row` is written (as tq_kv_write writes it, FP8 rows quantized) to pool row
 * page_table[seq_id[t]][pos[t] / 64] * 64 + pos[t] % 64.
 * rms(v) = v / sqrt(mean(v^2) + eps), computed in f32. rope rotates pairs (2i, 2i + 1) by the
 * angle pos * theta^(-2i / Dr) (angle reduced in f64). The projections are bf16 GEMMs with f32
 * accumulation: for T <= 128 the narrow ones (q_a and kv_a, at most one 128-row weight tile per
 * two SMs) on this library's weight-streaming tcgen05 kernel, the others on cuBLAS (opened at
 * run time as libcublas.so.12); the norms, RoPE, the assembly of q and the row writes are this
 * library's kernels.
 *   x        bf16 [T, Dm]              w_qa  bf16 [Rq, Dm]          q_norm  bf16 [Rq]
 *   w_qb     bf16 [H * (Dn + Dr), Rq]  w_uk  bf16 [H, Dn, 512]      w_kva   bf16 [W, Dm]
 *   kv_norm  bf16 [512]                pos, seq_id i32 [T]          page_table i32 [S, L]
 *   kv       u8 [P, 64, row bytes] pool of `kv_format` rows        q  bf16 [T, H, W] (out)
 * All matrices are packed row-major with 16-byte aligned bases; Dm, Rq and Dn are multiples of
 * 8. A row whose seq_id, pos or page entry is out of range is not written and sets
 * TQ_DEV_SEQ_RANGE, TQ_DEV_TABLE_SHORT or TQ_DEV_PAGE_RANGE in `device_flags` (a device int32,
 * may be null); its q is still produced. The workspace (tq_mla_prologue_workspace_bytes, 256-byte
 * aligned) holds the intermediates and cuBLAS's scratch; the first call on a device creates
 * that device's cuBLAS handle and the side stream on which the cache branch (kv_a projection,
 * RoPE, write) and then q's RoPE run beside the query branch (forked from and joined back into
 * `stream` with events), and the first call with a given token count asks the occupancy
 * calculator for the projection kernel's grid, so make those calls before capturing a stream.
 * Calls are serialised on
 * the host (one cuBLAS handle per device). No reference counterpart exists beyond the plan
 * line above. */
typedef struct {
  TqTensorSpec x, w_qa, q_norm, w_qb, w_uk, w_kva, kv_norm, pos, seq_id, page_table, kv, q;
  int32_t heads, nope_dim, rope_dim, kv_format;
  float q_eps, kv_eps, rope_theta;
} TqPrologueSpec;
int32_t tq_mla_prologue_validate(const TqPrologueSpec* spec, TqContractError* err);
int32_t tq_mla_prologue_workspace_bytes(const TqPrologueSpec* spec, uint64_t* bytes);
int32_t tq_mla_prologue(const TqPrologueSpec* spec, void* workspace, uint64_t workspace_bytes,
                        int32_t* device_flags, void* stream, TqContractError* err);

/* Measurement hook, no reference counterpart. Makes later tq_mla_decode / tq_mla_prefill calls
 * on the calling thread record `begin_event` right before and `end_event` right after the
 * attention kernel, on the launch stream (both are cudaEvent_t created by the caller). Pass two
 * nulls to switch it off; exactly one null is TQ_ERR_INVALID_ARGUMENT. */
int32_t tq_mla_set_kernel_timer(void* begin_event, void* end_event);

/* Philox4x32-10 test stream (host). tq_philox_words fills out[count]; an overflowing range
 * returns TQ_ERR_RANGE and leaves `out` untouched. */
void tq_philox_block(const uint32_t counter[4], const uint32_t key[2], uint32_t out[4]);
int32_t tq_philox_words(uint64_t seed, uint64_t stream_id, uint64_t start, uint32_t* out,
                        uint64_t count);
float tq_philox_uniform_f32(uint32_t word);

/* Seeded synthetic inputs on the device (Box-Muller normals rounded to bf16).
 *   tq_gen_normal_bf16: dst[i] = normal(seed, stream_id, start + i) for i < count.
 *   tq_gen_kv_pool: fills every row of the pool with NaN, then writes normal rows for each
 *   sequence's cached positions through the page table (normal index (tok_off[b]+p)*width+d). */
int32_t tq_gen_normal_bf16(void* dst, uint64_t count, uint64_t seed, uint64_t stream_id,
                           uint64_t start, void* stream);
int32_t tq_gen_kv_pool(void* pool, uint64_t pool_pages, uint64_t row_stride, uint64_t width,
                       const void* page_table, uint64_t slots, const void* kv_len,
                       const void* tok_off, uint64_t sequences, uint64_t seed, void* stream);

const char* tq_mla_status_string(int32_t status);
/* Library build identity: "tq_mla <version> sm_100a". */
const char* tq_mla_version(void);

#ifdef __cplusplus
}
#endif

#endif /* TQ_MLA_H */
