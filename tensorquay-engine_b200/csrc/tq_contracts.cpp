// Host contract validation for the dense paged MLA launch, and the Philox4x32-10 test stream.
//
// Validation restates SmlaParams::new (crates/tq-core/src/contracts.rs:437-493) and its helpers
// check (:262-325), check_strides (:331-356), check_kv_strides (:359-371) and check_aliases
// (:407-421): same field names, same violation kinds, same checked 64-bit span arithmetic, same
// empty-launch rule (docs/HOST-CONTRACTS.md:96-102). The generalisations (576-wide rows, 16/128
// heads, runtime scale for the 576 format, no sparse index tensors, f32 partial outputs,
// unbounded prefill plans) are listed in tq_contracts.h.
//
// Philox restates crates/tq-testkit/src/philox.rs:57-111 (block, fill_words, uniform_f32).

#include "tq_contracts.h"

#include <cmath>
#include <cstring>

namespace tq {

namespace {

constexpr uint64_t kDimensionLimit = uint64_t(1) << 31;
constexpr uint64_t kPageRows = 64;
constexpr uint64_t kKvGranularity = 16;
constexpr uint32_t kGlmScaleBits = 0x3D800000u;  // 0.0625f
constexpr uint64_t kDigestSalt = 0x7C3A5E1B9D2F4861ull;

enum class Layout { Packed, PaddedOuter, Checked };

struct Extent {
  const char* field;
  uint64_t start, end;
  bool present;
};

struct Failure {
  const char* field;
  int32_t kind;
};

uint64_t element_bytes(int32_t dtype) {
  switch (dtype) {
    case TQ_DTYPE_U8: return 1;
    case TQ_DTYPE_BF16: return 2;
    case TQ_DTYPE_I32:
    case TQ_DTYPE_F32: return 4;
    default: return 0;
  }
}

bool mul_overflows(uint64_t a, uint64_t b, uint64_t* out) {
  return __builtin_mul_overflow(a, b, out);
}
bool add_overflows(uint64_t a, uint64_t b, uint64_t* out) {
  return __builtin_add_overflow(a, b, out);
}

// Innermost stride is the element size; each outer stride spans the axis inside it.
bool check_strides(const TqTensorSpec& t, int rank, Layout layout, uint64_t element,
                   int32_t* kind) {
  if (t.strides_bytes[rank - 1] != element) { *kind = TQ_STRIDE; return false; }
  for (int axis = rank - 2; axis >= 0; --axis) {
    uint64_t inner = t.strides_bytes[axis + 1];
    uint64_t extent = t.shape[axis + 1] > 1 ? t.shape[axis + 1] : 1;
    uint64_t needed;
    if (mul_overflows(inner, extent, &needed)) { *kind = TQ_OVERFLOW; return false; }
    uint64_t stride = t.strides_bytes[axis];
    bool fits = layout == Layout::Packed ? stride == needed
                                         : (stride >= needed && stride % element == 0);
    if (!fits) { *kind = TQ_STRIDE; return false; }
  }
  return true;
}

// Checks one tensor; on success fills `ext` (present only when launching and non-empty).
bool check(const char* field, const TqTensorSpec& t, const uint64_t* shape, int rank,
           int32_t dtype, Layout layout, bool launching, Extent* ext, Failure* f) {
  ext->present = false;
  ext->field = field;
  if (t.rank != rank) { *f = {field, TQ_SHAPE}; return false; }
  if (t.dtype != dtype) { *f = {field, TQ_DTYPE}; return false; }
  for (int i = 0; i < rank; ++i)
    if (t.shape[i] != shape[i]) { *f = {field, TQ_SHAPE}; return false; }
  for (int i = 0; i < rank; ++i)
    if (t.shape[i] >= kDimensionLimit) { *f = {field, TQ_DIMENSION}; return false; }
  const uint64_t element = element_bytes(dtype);
  int32_t kind = 0;
  if (layout != Layout::Checked && !check_strides(t, rank, layout, element, &kind)) {
    *f = {field, kind};
    return false;
  }
  bool empty = false;
  for (int i = 0; i < rank; ++i) empty |= t.shape[i] == 0;
  if (!launching || empty) return true;
  uint64_t span = element;
  for (int i = 0; i < rank; ++i) {
    uint64_t reach;
    if (mul_overflows(t.shape[i] - 1, t.strides_bytes[i], &reach) ||
        add_overflows(span, reach, &span)) {
      *f = {field, TQ_OVERFLOW};
      return false;
    }
  }
  if (t.device_address == 0) { *f = {field, TQ_ADDRESS}; return false; }
  const uint64_t granularity = layout == Layout::Checked ? kKvGranularity : element;
  if (t.device_address % granularity != 0) { *f = {field, TQ_ALIGNMENT}; return false; }
  if (t.buffer_bytes < span) { *f = {field, TQ_CAPACITY}; return false; }
  uint64_t end;
  if (add_overflows(t.device_address, t.buffer_bytes, &end)) {
    *f = {field, TQ_OVERFLOW};
    return false;
  }
  // The bytes the tensor covers, not the capacity behind it (contracts.rs:318-324).
  *ext = {field, t.device_address, t.device_address + span, true};
  return true;
}

// Paged KV rows are [64 r, r, 1] with r at least the payload and a multiple of 16.
bool check_kv_strides(const TqTensorSpec& t, uint64_t payload, Failure* f) {
  if (t.rank != 3) { *f = {"kv", TQ_SHAPE}; return false; }
  const uint64_t row = t.strides_bytes[1];
  if (t.strides_bytes[2] != 1 || row < payload || row % kKvGranularity != 0) {
    *f = {"kv", TQ_STRIDE};
    return false;
  }
  uint64_t page;
  if (mul_overflows(kPageRows, row, &page)) { *f = {"kv", TQ_OVERFLOW}; return false; }
  if (t.strides_bytes[0] != page) { *f = {"kv", TQ_STRIDE}; return false; }
  return true;
}

bool check_aliases(const Extent* inputs, int n_in, const Extent* outputs, int n_out, Failure* f) {
  for (int o = 0; o < n_out; ++o) {
    const Extent& out = outputs[o];
    if (!out.present) continue;
    for (int i = 0; i < n_in + o; ++i) {
      const Extent& other = i < n_in ? inputs[i] : outputs[i - n_in];
      if (!other.present) continue;
      if (out.start < other.end && other.start < out.end) {
        *f = {out.field, TQ_ALIAS};
        return false;
      }
    }
  }
  return true;
}

uint32_t f32_bits(float x) {
  uint32_t b;
  std::memcpy(&b, &x, 4);
  return b;
}

bool scale_ok(int32_t format, float scale) {
  if (format == TQ_KV_BF16 || format == TQ_KV_FP8_E4M3) return f32_bits(scale) == kGlmScaleBits;
  return std::isfinite(scale) && scale > 0.0f;
}

// FNV-1a over the bytes of the params (digest field excluded).
uint64_t digest_of(const TqMlaParams& p) {
  const unsigned char* b = reinterpret_cast<const unsigned char*>(&p);
  const size_t n = offsetof(TqMlaParams, digest);
  uint64_t h = 0xCBF29CE484222325ull ^ kDigestSalt;
  for (size_t i = 0; i < n; ++i) {
    h ^= b[i];
    h *= 0x100000001B3ull;
  }
  return h;
}

template <typename Count>
// `idx` / `k_len` non-null: a sparse top-k plan (contracts.rs:442-470 checks them in this order:
// the index width right after q, then idx padded and k_len packed after kv_len).
int32_t validate_impl(const TqMlaSpec* spec, const Count* counts, uint64_t n, int max_per_seq,
                      TqMlaParams* params, TqContractError* err,
                      const TqTensorSpec* idx = nullptr, const TqTensorSpec* k_len = nullptr) {
  Failure f{nullptr, TQ_OK};
  auto fail = [&](const char* field, int32_t kind) {
    if (err) { err->field = field; err->kind = kind; }
    return kind;
  };
  if (!spec || (!counts && n != 0)) return fail("spec", TQ_ERR_INVALID_ARGUMENT);
  const TqMlaSpec& s = *spec;
  if (s.q.rank != 3) return fail("q", TQ_SHAPE);
  const uint64_t tokens = s.q.shape[0], heads = s.q.shape[1], width = s.q.shape[2];
  uint64_t payload = 0, qk_width = 0;
  switch (s.kv_format) {
    case TQ_KV_BF16: payload = 1024; qk_width = 512; break;
    case TQ_KV_FP8_E4M3: payload = 528; qk_width = 512; break;
    case TQ_KV_BF16_ROPE576: payload = 1152; qk_width = 576; break;
    default: return fail("kv_format", TQ_SHAPE);
  }
  if ((heads != 16 && heads != 32 && heads != 64 && heads != 128) || width != qk_width)
    return fail("q", TQ_SHAPE);
  const bool sparse = idx != nullptr;
  if (sparse && (!k_len || s.kv_format == TQ_KV_BF16_ROPE576)) return fail("kv_format", TQ_SHAPE);
  if (sparse && (idx->rank != 2 || idx->shape[1] > TQ_MLA_MAX_TOPK)) return fail("idx", TQ_SHAPE);
  if (!scale_ok(s.kv_format, s.softmax_scale)) return fail("softmax_scale", TQ_SCALE);
  if (s.page_table.rank != 2) return fail("page_table", TQ_SHAPE);
  const uint64_t sequences = s.page_table.shape[0], slots = s.page_table.shape[1];
  const bool launching = tokens != 0;
  if (!check_kv_strides(s.kv, payload, &f)) return fail(f.field, f.kind);

  const uint64_t query[3] = {tokens, heads, width};
  const uint64_t pool[3] = {s.kv.shape[0], kPageRows, payload};
  const uint64_t table[2] = {sequences, slots};
  const uint64_t tok[1] = {tokens};
  const uint64_t seqs[1] = {sequences};
  const uint64_t outshape[3] = {tokens, heads, 512};
  const uint64_t lseshape[2] = {tokens, heads};
  Extent in[8], out[2];
  if (!check("q", s.q, query, 3, TQ_DTYPE_BF16, Layout::PaddedOuter, launching, &in[0], &f) ||
      !check("kv", s.kv, pool, 3, TQ_DTYPE_U8, Layout::Checked, launching, &in[1], &f) ||
      !check("page_table", s.page_table, table, 2, TQ_DTYPE_I32, Layout::Packed, launching,
             &in[2], &f) ||
      !check("seq_id", s.seq_id, tok, 1, TQ_DTYPE_I32, Layout::Packed, launching, &in[3], &f) ||
      !check("q_pos", s.q_pos, tok, 1, TQ_DTYPE_I32, Layout::Packed, launching, &in[4], &f) ||
      !check("kv_len", s.kv_len, seqs, 1, TQ_DTYPE_I32, Layout::Packed, launching, &in[5], &f))
    return fail(f.field, f.kind);
  const uint64_t topk = sparse ? idx->shape[1] : 0;
  if (sparse) {
    const uint64_t idx_shape[2] = {tokens, topk};
    if (!check("idx", *idx, idx_shape, 2, TQ_DTYPE_I32, Layout::PaddedOuter, launching, &in[6],
               &f) ||
        !check("k_len", *k_len, tok, 1, TQ_DTYPE_I32, Layout::Packed, launching, &in[7], &f))
      return fail(f.field, f.kind);
  }
  // The output may be bf16 (final) or f32 (a partial result to merge across devices).
  const int32_t out_dtype = s.out.dtype == TQ_DTYPE_F32 ? TQ_DTYPE_F32 : TQ_DTYPE_BF16;
  if (!check("out", s.out, outshape, 3, out_dtype, Layout::PaddedOuter, launching, &out[0], &f) ||
      !check("lse", s.lse, lseshape, 2, TQ_DTYPE_F32, Layout::Packed, launching, &out[1], &f))
    return fail(f.field, f.kind);

  if (n != sequences) return fail("query_counts", TQ_QUERY_COUNT);
  uint64_t planned = 0;
  for (uint64_t i = 0; i < n; ++i) {
    const uint64_t c = counts[i];
    if (max_per_seq > 0 && c > uint64_t(max_per_seq)) return fail("query_counts", TQ_QUERY_COUNT);
    planned += c;  // n < 2^31 and c < 2^32: cannot wrap
  }
  if (planned != tokens) return fail("query_counts", TQ_QUERY_COUNT);
  if (!check_aliases(in, sparse ? 8 : 6, out, 2, &f)) return fail(f.field, f.kind);

  if (params) {
    std::memset(params, 0, sizeof(*params));
    params->spec = s;
    params->tokens = tokens;
    params->heads = heads;
    params->sequences = sequences;
    params->slots = slots;
    params->pages = s.kv.shape[0];
    params->qk_width = qk_width;
    params->row_stride = s.kv.strides_bytes[1];
    params->max_queries_per_sequence = max_per_seq;
    params->should_launch = launching ? 1 : 0;
    if (sparse) {
      params->idx = *idx;
      params->k_len = *k_len;
      params->topk = topk;
      params->sparse = 1;
    }
    params->digest = digest_of(*params);
  }
  if (err) { err->field = nullptr; err->kind = TQ_OK; }
  return TQ_OK;
}

// The KV writer's declarations: the same per-tensor checks as the attention plan, the pool as
// the output that no input may overlap, and 16-byte vector access to the source rows.
int32_t kv_write_validate_impl(const TqKvWriteSpec* spec, TqContractError* err) {
  Failure f{nullptr, TQ_OK};
  auto fail = [&](const char* field, int32_t kind) {
    if (err) { err->field = field; err->kind = kind; }
    return kind;
  };
  if (!spec) return fail("spec", TQ_ERR_INVALID_ARGUMENT);
  const TqKvWriteSpec& s = *spec;
  uint64_t payload = 0, width = 0;
  switch (s.kv_format) {
    case TQ_KV_BF16: payload = 1024; width = 512; break;
    case TQ_KV_FP8_E4M3: payload = 528; width = 512; break;
    case TQ_KV_BF16_ROPE576: payload = 1152; width = 576; break;
    default: return fail("kv_format", TQ_SHAPE);
  }
  if (s.src.rank != 2) return fail("src", TQ_SHAPE);
  if (s.page_table.rank != 2) return fail("page_table", TQ_SHAPE);
  const uint64_t rows = s.src.shape[0];
  const uint64_t sequences = s.page_table.shape[0], slots = s.page_table.shape[1];
  const bool launching = rows != 0;
  if (!check_kv_strides(s.kv, payload, &f)) return fail(f.field, f.kind);
  const uint64_t src_shape[2] = {rows, width};
  const uint64_t pool[3] = {s.kv.shape[0], kPageRows, payload};
  const uint64_t table[2] = {sequences, slots};
  const uint64_t tok[1] = {rows};
  Extent in[5], out[1];
  if (!check("src", s.src, src_shape, 2, TQ_DTYPE_BF16, Layout::PaddedOuter, launching, &in[0],
             &f) ||
      !check("page_table", s.page_table, table, 2, TQ_DTYPE_I32, Layout::Packed, launching,
             &in[1], &f) ||
      !check("seq_id", s.seq_id, tok, 1, TQ_DTYPE_I32, Layout::Packed, launching, &in[2], &f) ||
      !check("pos", s.pos, tok, 1, TQ_DTYPE_I32, Layout::Packed, launching, &in[3], &f) ||
      !check("kv", s.kv, pool, 3, TQ_DTYPE_U8, Layout::Checked, launching, &out[0], &f))
    return fail(f.field, f.kind);
  if (launching) {
    if (s.src.strides_bytes[0] % 16) return fail("src", TQ_STRIDE);
    if (s.src.device_address % 16) return fail("src", TQ_ALIGNMENT);
  }
  int n_in = 4;
  if (s.norm_weight.rank != 0) {
    const uint64_t w_shape[1] = {512};
    if (!check("norm_weight", s.norm_weight, w_shape, 1, TQ_DTYPE_BF16, Layout::Packed,
               launching, &in[4], &f))
      return fail(f.field, f.kind);
    if (launching && s.norm_weight.device_address % 16) return fail("norm_weight", TQ_ALIGNMENT);
    if (!(std::isfinite(s.norm_eps) && s.norm_eps > 0.f)) return fail("norm_eps", TQ_SCALE);
    n_in = 5;
  }
  if (!check_aliases(in, n_in, out, 1, &f)) return fail(f.field, f.kind);
  if (err) { err->field = nullptr; err->kind = TQ_OK; }
  return TQ_OK;
}

// MLA prologue: the same tensor-declaration rules (shape, dtype, packed strides, spans, null,
// alignment, capacity; outputs never alias inputs), plus 16-byte aligned rows for the GEMMs.
int32_t prologue_validate_impl(const TqPrologueSpec* spec, TqContractError* err) {
  Failure f{nullptr, TQ_OK};
  auto fail = [&](const char* field, int32_t kind) {
    if (err) { err->field = field; err->kind = kind; }
    return kind;
  };
  if (!spec) return fail("spec", TQ_ERR_INVALID_ARGUMENT);
  const TqPrologueSpec& s = *spec;
  if (s.x.rank != 2) return fail("x", TQ_SHAPE);
  if (s.w_qa.rank != 2) return fail("w_qa", TQ_SHAPE);
  if (s.page_table.rank != 2) return fail("page_table", TQ_SHAPE);
  if (s.heads <= 0 || s.heads > 128) return fail("heads", TQ_SHAPE);
  if (s.nope_dim <= 0 || s.nope_dim > 512 || s.nope_dim % 8) return fail("nope_dim", TQ_SHAPE);
  if (s.rope_dim != 0 && s.rope_dim != 64) return fail("rope_dim", TQ_SHAPE);
  uint64_t payload = 0;
  switch (s.kv_format) {
    case TQ_KV_BF16: payload = 1024; break;
    case TQ_KV_FP8_E4M3: payload = 528; break;
    case TQ_KV_BF16_ROPE576: payload = 1152; break;
    default: return fail("kv_format", TQ_SHAPE);
  }
  if ((s.kv_format == TQ_KV_BF16_ROPE576) != (s.rope_dim == 64)) return fail("kv_format", TQ_SHAPE);
  const uint64_t T = s.x.shape[0], dm = s.x.shape[1], rq = s.w_qa.shape[0];
  const uint64_t H = uint64_t(s.heads), dn = uint64_t(s.nope_dim), dr = uint64_t(s.rope_dim);
  if (dm == 0 || dm % 8 || dm > (1u << 20)) return fail("x", TQ_SHAPE);
  if (rq == 0 || rq % 8 || rq > (1u << 16)) return fail("w_qa", TQ_SHAPE);
  if (T > (1u << 24)) return fail("x", TQ_SHAPE);
  const bool launching = T != 0;
  if (!check_kv_strides(s.kv, payload, &f)) return fail(f.field, f.kind);
  const uint64_t x_shape[2] = {T, dm}, wqa[2] = {rq, dm}, qn[1] = {rq};
  const uint64_t wqb[2] = {H * (dn + dr), rq}, wuk[3] = {H, dn, 512}, wkva[2] = {512 + dr, dm};
  const uint64_t kvn[1] = {512}, tok[1] = {T};
  const uint64_t table[2] = {s.page_table.shape[0], s.page_table.shape[1]};
  const uint64_t pool[3] = {s.kv.shape[0], kPageRows, payload}, q_shape[3] = {T, H, 512 + dr};
  Extent in[10], out[2];
  if (!check("x", s.x, x_shape, 2, TQ_DTYPE_BF16, Layout::Packed, launching, &in[0], &f) ||
      !check("w_qa", s.w_qa, wqa, 2, TQ_DTYPE_BF16, Layout::Packed, launching, &in[1], &f) ||
      !check("q_norm", s.q_norm, qn, 1, TQ_DTYPE_BF16, Layout::Packed, launching, &in[2], &f) ||
      !check("w_qb", s.w_qb, wqb, 2, TQ_DTYPE_BF16, Layout::Packed, launching, &in[3], &f) ||
      !check("w_uk", s.w_uk, wuk, 3, TQ_DTYPE_BF16, Layout::Packed, launching, &in[4], &f) ||
      !check("w_kva", s.w_kva, wkva, 2, TQ_DTYPE_BF16, Layout::Packed, launching, &in[5], &f) ||
      !check("kv_norm", s.kv_norm, kvn, 1, TQ_DTYPE_BF16, Layout::Packed, launching, &in[6], &f) ||
      !check("pos", s.pos, tok, 1, TQ_DTYPE_I32, Layout::Packed, launching, &in[7], &f) ||
      !check("seq_id", s.seq_id, tok, 1, TQ_DTYPE_I32, Layout::Packed, launching, &in[8], &f) ||
      !check("page_table", s.page_table, table, 2, TQ_DTYPE_I32, Layout::Packed, launching,
             &in[9], &f) ||
      !check("kv", s.kv, pool, 3, TQ_DTYPE_U8, Layout::Checked, launching, &out[0], &f) ||
      !check("q", s.q, q_shape, 3, TQ_DTYPE_BF16, Layout::Packed, launching, &out[1], &f))
    return fail(f.field, f.kind);
  if (launching) {
    const TqTensorSpec* mats[8] = {&s.x, &s.w_qa, &s.q_norm, &s.w_qb, &s.w_uk, &s.w_kva,
                                   &s.kv_norm, &s.q};
    const char* names[8] = {"x", "w_qa", "q_norm", "w_qb", "w_uk", "w_kva", "kv_norm", "q"};
    for (int i = 0; i < 8; ++i)
      if (mats[i]->device_address % 16) return fail(names[i], TQ_ALIGNMENT);
  }
  if (!(std::isfinite(s.q_eps) && s.q_eps > 0.f)) return fail("q_eps", TQ_SCALE);
  if (!(std::isfinite(s.kv_eps) && s.kv_eps > 0.f)) return fail("kv_eps", TQ_SCALE);
  if (!(std::isfinite(s.rope_theta) && s.rope_theta > 1.f)) return fail("rope_theta", TQ_SCALE);
  if (!check_aliases(in, 10, out, 2, &f)) return fail(f.field, f.kind);
  if (err) { err->field = nullptr; err->kind = TQ_OK; }
  return TQ_OK;
}

}  // namespace

int32_t prologue_validate(const TqPrologueSpec* spec, TqContractError* err) {
  return prologue_validate_impl(spec, err);
}

bool params_intact(const TqMlaParams* p) { return p && p->digest == digest_of(*p); }

// ---------------------------------------------------------------------------------------------
// Philox4x32-10: ten rounds, key bumped by (W0, W1) per round (philox.rs:57-70).

void philox_block(const uint32_t counter[4], const uint32_t key[2], uint32_t out[4]) {
  uint32_t c0 = counter[0], c1 = counter[1], c2 = counter[2], c3 = counter[3];
  uint32_t k0 = key[0], k1 = key[1];
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = uint64_t(0xD2511F53u) * c0;
    const uint64_t p1 = uint64_t(0xCD9E8D57u) * c2;
    const uint32_t n0 = uint32_t(p1 >> 32) ^ c1 ^ k0;
    const uint32_t n2 = uint32_t(p0 >> 32) ^ c3 ^ k1;
    c1 = uint32_t(p1);
    c3 = uint32_t(p0);
    c0 = n0;
    c2 = n2;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

int32_t philox_words(uint64_t seed, uint64_t stream, uint64_t start, uint32_t* out,
                     uint64_t count) {
  if (count == 0) return TQ_OK;
  uint64_t last;
  if (add_overflows(start, count - 1, &last)) return TQ_ERR_RANGE;
  if (!out) return TQ_ERR_INVALID_ARGUMENT;
  const uint32_t key[2] = {uint32_t(seed), uint32_t(seed >> 32)};
  uint64_t i = start, written = 0;
  while (written < count) {
    const uint64_t group = i >> 2;
    const uint32_t counter[4] = {uint32_t(group), uint32_t(group >> 32), uint32_t(stream),
                                 uint32_t(stream >> 32)};
    uint32_t lanes[4];
    philox_block(counter, key, lanes);
    for (unsigned lane = unsigned(i & 3); lane < 4 && written < count; ++lane) {
      out[written++] = lanes[lane];
      ++i;
    }
  }
  return TQ_OK;
}

float philox_uniform_f32(uint32_t word) { return float(word >> 8) * (1.0f / 16777216.0f); }

}  // namespace tq

extern "C" {

int32_t tq_mla_validate(const TqMlaSpec* spec, const uint8_t* query_counts, uint64_t n,
                        TqMlaParams* params, TqContractError* err) {
  return tq::validate_impl(spec, query_counts, n, 4, params, err);
}

int32_t tq_mla_prefill_validate(const TqMlaSpec* spec, const uint32_t* query_counts, uint64_t n,
                                TqMlaParams* params, TqContractError* err) {
  return tq::validate_impl(spec, query_counts, n, 0, params, err);
}

int32_t tq_mla_sparse_validate(const TqMlaSpec* spec, const TqTensorSpec* idx,
                               const TqTensorSpec* k_len, const uint8_t* query_counts, uint64_t n,
                               TqMlaParams* params, TqContractError* err) {
  if (!idx || !k_len) {
    if (err) { err->field = "idx"; err->kind = TQ_ERR_INVALID_ARGUMENT; }
    return TQ_ERR_INVALID_ARGUMENT;
  }
  return tq::validate_impl(spec, query_counts, n, 4, params, err, idx, k_len);
}

int32_t tq_kv_write_validate(const TqKvWriteSpec* spec, TqContractError* err) {
  return tq::kv_write_validate_impl(spec, err);
}

int32_t tq_mla_prologue_validate(const TqPrologueSpec* spec, TqContractError* err) {
  return tq::prologue_validate(spec, err);
}

int32_t tq_mla_should_launch(const TqMlaParams* params) {
  return tq::params_intact(params) ? params->should_launch : 0;
}

void tq_philox_block(const uint32_t counter[4], const uint32_t key[2], uint32_t out[4]) {
  tq::philox_block(counter, key, out);
}

int32_t tq_philox_words(uint64_t seed, uint64_t stream_id, uint64_t start, uint32_t* out,
                        uint64_t count) {
  return tq::philox_words(seed, stream_id, start, out, count);
}

float tq_philox_uniform_f32(uint32_t word) { return tq::philox_uniform_f32(word); }

const char* tq_mla_status_string(int32_t status) {
  switch (status) {
    case TQ_OK: return "ok";
    case TQ_SHAPE: return "Shape";
    case TQ_DTYPE: return "Dtype";
    case TQ_DIMENSION: return "Dimension";
    case TQ_STRIDE: return "Stride";
    case TQ_ALIGNMENT: return "Alignment";
    case TQ_ADDRESS: return "Address";
    case TQ_CAPACITY: return "Capacity";
    case TQ_OVERFLOW: return "Overflow";
    case TQ_QUERY_COUNT: return "QueryCount";
    case TQ_SCALE: return "Scale";
    case TQ_GROUP: return "Group";
    case TQ_ALIAS: return "Alias";
    case TQ_ERR_INVALID_ARGUMENT: return "invalid argument";
    case TQ_ERR_UNSUPPORTED: return "unsupported layout";
    case TQ_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case TQ_ERR_CUDA: return "CUDA error";
    case TQ_ERR_PARAMS: return "params not produced by validation";
    case TQ_ERR_RANGE: return "word range exceeds u64";
    case TQ_ERR_COMM: return "NCCL unavailable or a collective failed";
    default: return "unknown status";
  }
}

}  // extern "C"
