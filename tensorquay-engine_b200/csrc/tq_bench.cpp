// tq_bench: native benchmark of the paged-MLA path through the C ABI alone (include/tq_mla.h).
//
// The reference plans a benchmark binary (`tq-bench`, docs/ARCHITECTURE.md:56) with the timing
// protocol of docs/TEST-PLAN.md:341-360: warm-up, at least 50 timed runs, median / p10 / p90 /
// IQR, device timing with events, optional graph replay. This is that binary for the dense
// paged path. It links libtq_mla.so and the CUDA runtime only (no Python, no PyTorch).
//
// Inputs are the seeded configurations of the library's generator: host metadata (lengths,
// page permutation, block tables, token-balanced shards) is drawn here from the library's
// Philox stream (tq_philox_words) with the same transforms as the Python host mirror, and the
// device data (queries, cache rows) by tq_gen_normal_bf16 / tq_gen_kv_pool. So a batch is the
// same, bit for bit, whichever front end builds it.
//
// Usage: tq_bench [--config decode|prefill|longctx|mtp|cpu] [--steps K] [--warmup W]
//                 [--runs R] [--steps-per-run S] [--world N --rank r] [--strong]
//                 [--graph] [--dump-out FILE] [--dump-meta]
// One JSON line on stdout. --dump-meta prints the host metadata as JSON and touches no GPU.

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <numeric>
#include <string>
#include <vector>

#include "../../include/tq_mla.h"

namespace {

constexpr int kPageRows = 64;
constexpr uint64_t kStreamQ = 1, kStreamLen = 3, kStreamPerm = 4, kStreamPrefix = 5;

[[noreturn]] void die(const char* what, long long code) {
  std::fprintf(stderr, "tq_bench: %s (%lld)\n", what, code);
  std::exit(1);
}

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) die(cudaGetErrorString(e), int(e));
  (void)what;
}

void ckt(int32_t st, const char* what) {
  if (st != TQ_OK) {
    std::fprintf(stderr, "tq_bench: %s: %s\n", what, tq_mla_status_string(st));
    std::exit(1);
  }
}

std::vector<uint32_t> words(uint64_t seed, uint64_t stream, uint64_t start, uint64_t count) {
  std::vector<uint32_t> w(std::max<uint64_t>(count, 1));
  ckt(tq_philox_words(seed, stream, start, w.data(), count), "philox");
  w.resize(count);
  return w;
}

std::vector<int64_t> bounded(uint64_t seed, uint64_t stream, int count, int64_t lo, int64_t hi) {
  const auto w = words(seed, stream, 0, count);
  std::vector<int64_t> v(count);
  for (int i = 0; i < count; ++i) v[i] = lo + int64_t(w[i]) % (hi - lo + 1);
  return v;
}

// Normal i of a stream: Box-Muller on words 2i and 2i+1 (the generator's transform).
std::vector<double> normals(uint64_t seed, uint64_t stream, int count) {
  const auto w = words(seed, stream, 0, 2 * uint64_t(count));
  std::vector<double> z(count);
  for (int i = 0; i < count; ++i) {
    const double u1 = (double(w[2 * i] >> 8) + 1.0) * std::ldexp(1.0, -24);
    const double u2 = double(w[2 * i + 1] >> 8) * std::ldexp(1.0, -24);
    z[i] = std::sqrt(-2.0 * std::log(u1)) * std::cos(2.0 * M_PI * u2);
  }
  return z;
}

std::vector<int64_t> permutation(uint64_t seed, int64_t pages) {
  std::vector<int64_t> perm(pages);
  std::iota(perm.begin(), perm.end(), 0);
  if (pages > 1) {
    const auto w = words(seed, kStreamPerm, 0, pages - 1);
    for (int64_t k = 0; k < pages - 1; ++k) {
      const int64_t i = pages - 1 - k, j = int64_t(w[k]) % (i + 1);
      std::swap(perm[i], perm[j]);
    }
  }
  return perm;
}

struct Workload {
  std::string name;
  uint64_t seed = 0;
  int heads = 0, width = 0;
  float scale = 0.f;
  bool prefill = false;
  std::vector<int64_t> kv_len, q_per_seq, prefix, token_global, tok_off_global;
  std::vector<int32_t> page_table;  // [S, slots]
  int64_t slots = 1, pool_pages = 0;

  int64_t sequences() const { return int64_t(kv_len.size()); }
  int64_t tokens() const { return std::accumulate(q_per_seq.begin(), q_per_seq.end(), int64_t(0)); }
  double visible_sum() const {
    double v = 0;
    for (size_t b = 0; b < kv_len.size(); ++b)
      for (int64_t i = 0; i < q_per_seq[b]; ++i) v += double(std::min(kv_len[b], prefix[b] + i + 1));
    return v;
  }
  double flops() const { return 2.0 * heads * (width + 512) * visible_sum(); }
  double bytes() const {
    double rows = 0, pages = 0;
    for (auto n : kv_len) {
      rows += double(n);
      pages += double((n + kPageRows - 1) / kPageRows);
    }
    return rows * width * 2 + double(tokens()) * heads * (width * 2 + 1024 + 4) + 4 * pages +
           4 * double(sequences());
  }
};

std::vector<int64_t> exclusive_sum(const std::vector<int64_t>& v) {
  std::vector<int64_t> o(v.size(), 0);
  for (size_t i = 1; i < v.size(); ++i) o[i] = o[i - 1] + v[i - 1];
  return o;
}

// Block tables from a permuted pool holding exactly the cached pages (or `pool` pages).
void finish(Workload& w, int64_t pool = -1) {
  std::vector<int64_t> np(w.kv_len.size());
  int64_t total = 0, width = 1;
  for (size_t b = 0; b < np.size(); ++b) {
    np[b] = (w.kv_len[b] + kPageRows - 1) / kPageRows;
    total += np[b];
    width = std::max(width, np[b]);
  }
  w.pool_pages = pool < 0 ? total : pool;
  if (w.pool_pages < total) die("pool smaller than the cached pages", w.pool_pages);
  const auto perm = permutation(w.seed, w.pool_pages);
  w.slots = width;
  w.page_table.assign(np.size() * width, 0);
  int64_t off = 0;
  for (size_t b = 0; b < np.size(); ++b)
    for (int64_t i = 0; i < np[b]; ++i) w.page_table[b * width + i] = int32_t(perm[off++]);
  if (w.token_global.empty()) w.token_global = exclusive_sum(w.q_per_seq);
  if (w.tok_off_global.empty()) w.tok_off_global = exclusive_sum(w.kv_len);
}

Workload config(const std::string& name, int batch) {
  Workload w;
  const float s576 = float(1.0 / std::sqrt(192.0));
  auto ones = [](int b) { return std::vector<int64_t>(b, 1); };
  if (name == "cpu") {
    w = Workload{"cpu_decode_h16", 0, 16, 576, s576};
    w.kv_len = {17, 64, 200, 1000};
    w.q_per_seq = ones(4);
    for (auto n : w.kv_len) w.prefix.push_back(n - 1);
    finish(w, 64);
    return w;
  }
  if (name == "decode") {
    const int b = batch > 0 ? batch : 64;
    w = Workload{"decode_b64_h128_ctx4k-8k", 1, 128, 576, s576};
    w.kv_len = bounded(1, kStreamLen, b, 4096, 8192);
    w.q_per_seq = ones(b);
  } else if (name == "prefill") {
    const int b = batch > 0 ? batch : 8;
    w = Workload{"prefill_8x2048_prefix0-6k_h128", 2, 128, 576, s576, true};
    const auto pre = bounded(2, kStreamPrefix, b, 0, 6144);
    for (auto p : pre) w.kv_len.push_back(p + 2048);
    w.q_per_seq.assign(b, 2048);
    w.prefix = pre;
    finish(w);
    return w;
  } else if (name == "longctx") {
    const int b = batch > 0 ? batch : 4;
    w = Workload{"longctx_b4_131072_h128", 3, 128, 576, s576};
    w.kv_len.assign(b, 131072);
    w.q_per_seq = ones(b);
  } else if (name == "mtp") {
    const int b = batch > 0 ? batch : 512;
    w = Workload{"mtp_512x2_lognormal8k_h128", 4, 128, 576, s576};
    const auto z = normals(4, kStreamLen, b);
    for (int i = 0; i < b; ++i) {
      const double v = std::nearbyint(std::exp(std::log(8192.0) + 1.0 * z[i]));
      w.kv_len.push_back(int64_t(std::min(65536.0, std::max(256.0, v))));
    }
    w.q_per_seq.assign(b, 2);
    for (auto n : w.kv_len) w.prefix.push_back(n - 2);
    finish(w);
    return w;
  } else {
    die("unknown --config", 0);
  }
  for (auto n : w.kv_len) w.prefix.push_back(n - 1);
  finish(w);
  return w;
}

// Token-balanced (longest-first greedy) share of whole sequences for rank `rank` of `world`.
Workload shard(const Workload& w, int world, int rank) {
  const int64_t S = w.sequences();
  std::vector<int64_t> cost(S), order(S);
  for (int64_t b = 0; b < S; ++b) cost[b] = w.kv_len[b] * w.q_per_seq[b];
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int64_t a, int64_t b) { return cost[a] > cost[b]; });
  std::vector<double> load(world, 0.0);
  std::vector<int> owner(S, 0);
  for (auto b : order) {
    const int r = int(std::min_element(load.begin(), load.end()) - load.begin());
    owner[b] = r;
    load[r] += double(cost[b]);
  }
  const auto tok_global = exclusive_sum(w.q_per_seq), tok_off = exclusive_sum(w.kv_len);
  Workload s;
  s.name = w.name;
  s.seed = w.seed;
  s.heads = w.heads;
  s.width = w.width;
  s.scale = w.scale;
  s.prefill = w.prefill;
  for (int64_t b = 0; b < S; ++b) {
    if (owner[b] != rank) continue;
    s.kv_len.push_back(w.kv_len[b]);
    s.q_per_seq.push_back(w.q_per_seq[b]);
    s.prefix.push_back(w.prefix[b]);
    s.token_global.push_back(tok_global[b]);
    s.tok_off_global.push_back(tok_off[b]);
  }
  finish(s);
  return s;
}

template <typename T>
void print_array(const char* key, const std::vector<T>& v, bool last = false) {
  std::printf("\"%s\": [", key);
  for (size_t i = 0; i < v.size(); ++i) std::printf("%s%lld", i ? ", " : "", (long long)v[i]);
  std::printf("]%s", last ? "" : ", ");
}

TqTensorSpec spec(std::initializer_list<uint64_t> shape, std::initializer_list<uint64_t> strides,
                  int32_t dtype, const void* addr, uint64_t bytes) {
  TqTensorSpec t;
  std::memset(&t, 0, sizeof(t));
  t.rank = int32_t(shape.size());
  int i = 0;
  for (auto d : shape) t.shape[i++] = d;
  i = 0;
  for (auto s : strides) t.strides_bytes[i++] = s;
  t.dtype = dtype;
  t.device_address = reinterpret_cast<uint64_t>(addr);
  t.buffer_bytes = bytes;
  return t;
}

struct Stats {
  double p10, p25, median, p75, p90, mean;
};

Stats stats_of(std::vector<double> v) {
  std::sort(v.begin(), v.end());
  auto q = [&](double p) {  // linear interpolation between order statistics
    const double x = p * double(v.size() - 1);
    const size_t i = size_t(x);
    const double f = x - double(i);
    return i + 1 < v.size() ? v[i] * (1 - f) + v[i + 1] * f : v[i];
  };
  return {q(0.10), q(0.25), q(0.50), q(0.75), q(0.90),
          std::accumulate(v.begin(), v.end(), 0.0) / double(v.size())};
}

struct Device {
  void* q = nullptr;
  void* kv = nullptr;
  void* meta = nullptr;  // page_table | seq_id | q_pos | kv_len, each 16-byte aligned
  void* out = nullptr;
  void* lse = nullptr;
  uint64_t q_bytes = 0, kv_bytes = 0, meta_bytes = 0, out_bytes = 0, lse_bytes = 0;
  uint64_t off_pt = 0, off_seq = 0, off_qpos = 0, off_kvlen = 0;
};

uint64_t up16(uint64_t x) { return (x + 15) & ~uint64_t(15); }

}  // namespace

int main(int argc, char** argv) {
  std::string cfg = "decode", dump_out;
  int steps = 1000, warmup = 10, runs = 50, per_run = 10, world = 1, rank = 0, device = 0;
  bool graph = false, dump_meta = false, strong = false;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto next = [&]() -> const char* {
      if (i + 1 >= argc) die("missing value", i);
      return argv[++i];
    };
    if (a == "--config") cfg = next();
    else if (a == "--steps") steps = std::atoi(next());
    else if (a == "--warmup") warmup = std::atoi(next());
    else if (a == "--runs") runs = std::atoi(next());
    else if (a == "--steps-per-run") per_run = std::atoi(next());
    else if (a == "--world") world = std::atoi(next());
    else if (a == "--rank") rank = std::atoi(next());
    else if (a == "--device") device = std::atoi(next());
    else if (a == "--strong") strong = true;
    else if (a == "--graph") graph = true;
    else if (a == "--dump-out") dump_out = next();
    else if (a == "--dump-meta") dump_meta = true;
    else die("unknown argument", i);
  }
  if (steps < 1 || warmup < 0 || runs < 1 || per_run < 1 || world < 1 || rank < 0 || rank >= world)
    die("bad counts", 0);
  static const int base_batch[] = {64, 8, 4, 512};
  const char* names[] = {"decode", "prefill", "longctx", "mtp"};
  int batch = 0;
  if (!strong && world > 1)
    for (int k = 0; k < 4; ++k)
      if (cfg == names[k]) batch = base_batch[k] * world;
  const Workload full = config(cfg, batch);
  const Workload w = world > 1 ? shard(full, world, rank) : full;
  const int64_t T = w.tokens(), S = w.sequences(), H = w.heads, D = w.width;

  if (dump_meta) {
    std::printf("{\"name\": \"%s\", \"seed\": %llu, \"heads\": %d, \"width\": %d, \"scale\": %.9g, ",
                w.name.c_str(), (unsigned long long)w.seed, w.heads, w.width, double(w.scale));
    std::printf("\"pool_pages\": %lld, \"slots\": %lld, ", (long long)w.pool_pages,
                (long long)w.slots);
    print_array("kv_len", w.kv_len);
    print_array("q_per_seq", w.q_per_seq);
    print_array("prefix", w.prefix);
    print_array("token_global", w.token_global);
    print_array("tok_off_global", w.tok_off_global);
    print_array("page_table", w.page_table, true);
    std::printf("}\n");
    return 0;
  }

  ck(cudaSetDevice(device), "device");
  cudaStream_t st, s_in, s_out;
  ck(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "stream");
  ck(cudaStreamCreateWithFlags(&s_in, cudaStreamNonBlocking), "stream");
  ck(cudaStreamCreateWithFlags(&s_out, cudaStreamNonBlocking), "stream");

  // ---- host metadata and device inputs
  std::vector<int32_t> seq_id, q_pos, kv_len32(w.kv_len.begin(), w.kv_len.end());
  for (int64_t b = 0; b < S; ++b)
    for (int64_t i = 0; i < w.q_per_seq[b]; ++i) {
      seq_id.push_back(int32_t(b));
      q_pos.push_back(int32_t(w.prefix[b] + i));
    }
  const uint64_t row = uint64_t(D) * 2;
  auto alloc_set = [&](Device& d, bool with_kv, const Device* share) {
    d.q_bytes = std::max<uint64_t>(uint64_t(T) * H * D * 2, 16);
    d.off_pt = 0;
    d.off_seq = up16(w.page_table.size() * 4);
    d.off_qpos = d.off_seq + up16(T * 4);
    d.off_kvlen = d.off_qpos + up16(T * 4);
    d.meta_bytes = d.off_kvlen + up16(S * 4);
    d.out_bytes = std::max<uint64_t>(uint64_t(T) * H * 512 * 2, 16);
    d.lse_bytes = std::max<uint64_t>(uint64_t(T) * H * 4, 16);
    ck(cudaMalloc(&d.q, d.q_bytes), "q");
    ck(cudaMalloc(&d.meta, d.meta_bytes), "meta");
    ck(cudaMalloc(&d.out, d.out_bytes), "out");
    ck(cudaMalloc(&d.lse, d.lse_bytes), "lse");
    if (with_kv) {
      d.kv_bytes = std::max<uint64_t>(uint64_t(w.pool_pages) * kPageRows * row, 16);
      ck(cudaMalloc(&d.kv, d.kv_bytes), "kv");
    } else {
      d.kv = share->kv;
      d.kv_bytes = share->kv_bytes;
    }
  };
  std::vector<uint8_t> h_meta_buf;
  Device dev;
  alloc_set(dev, true, nullptr);
  h_meta_buf.assign(dev.meta_bytes, 0);
  std::memcpy(h_meta_buf.data() + dev.off_pt, w.page_table.data(), w.page_table.size() * 4);
  std::memcpy(h_meta_buf.data() + dev.off_seq, seq_id.data(), T * 4);
  std::memcpy(h_meta_buf.data() + dev.off_qpos, q_pos.data(), T * 4);
  std::memcpy(h_meta_buf.data() + dev.off_kvlen, kv_len32.data(), S * 4);
  ck(cudaMemcpy(dev.meta, h_meta_buf.data(), dev.meta_bytes, cudaMemcpyHostToDevice), "meta");
  {
    int64_t local = 0;
    for (int64_t b = 0; b < S; ++b) {
      const uint64_t n = uint64_t(w.q_per_seq[b]) * H * D;
      if (n)
        ckt(tq_gen_normal_bf16(static_cast<uint16_t*>(dev.q) + uint64_t(local) * H * D, n, w.seed,
                               kStreamQ, uint64_t(w.token_global[b]) * H * D, st),
            "gen q");
      local += w.q_per_seq[b];
    }
    void* tok_off = nullptr;
    ck(cudaMalloc(&tok_off, std::max<size_t>(S * 8, 8)), "tok_off");
    ck(cudaMemcpy(tok_off, w.tok_off_global.data(), S * 8, cudaMemcpyHostToDevice), "tok_off");
    ckt(tq_gen_kv_pool(dev.kv, w.pool_pages, row, D, static_cast<char*>(dev.meta) + dev.off_pt,
                       w.slots, static_cast<char*>(dev.meta) + dev.off_kvlen, tok_off, S, w.seed,
                       st),
        "gen kv");
    ck(cudaStreamSynchronize(st), "gen");
    ck(cudaFree(tok_off), "free");
  }

  // ---- validated launches (one per buffer set) and their workspaces
  auto make_params = [&](const Device& d, TqMlaParams* p) {
    TqMlaSpec s;
    std::memset(&s, 0, sizeof(s));
    s.q = spec({uint64_t(T), uint64_t(H), uint64_t(D)}, {uint64_t(H * D * 2), uint64_t(D * 2), 2},
               TQ_DTYPE_BF16, d.q, d.q_bytes);
    s.kv = spec({uint64_t(w.pool_pages), kPageRows, row}, {kPageRows * row, row, 1}, TQ_DTYPE_U8,
                d.kv, d.kv_bytes);
    s.page_table = spec({uint64_t(S), uint64_t(w.slots)}, {uint64_t(w.slots) * 4, 4}, TQ_DTYPE_I32,
                        static_cast<char*>(d.meta) + d.off_pt, w.page_table.size() * 4);
    s.seq_id = spec({uint64_t(T)}, {4}, TQ_DTYPE_I32, static_cast<char*>(d.meta) + d.off_seq, T * 4);
    s.q_pos = spec({uint64_t(T)}, {4}, TQ_DTYPE_I32, static_cast<char*>(d.meta) + d.off_qpos, T * 4);
    s.kv_len = spec({uint64_t(S)}, {4}, TQ_DTYPE_I32, static_cast<char*>(d.meta) + d.off_kvlen, S * 4);
    s.out = spec({uint64_t(T), uint64_t(H), 512}, {uint64_t(H * 1024), 1024, 2}, TQ_DTYPE_BF16, d.out,
                 d.out_bytes);
    s.lse = spec({uint64_t(T), uint64_t(H)}, {uint64_t(H * 4), 4}, TQ_DTYPE_F32, d.lse, d.lse_bytes);
    s.kv_format = D == 576 ? TQ_KV_BF16_ROPE576 : TQ_KV_BF16;
    s.softmax_scale = w.scale;
    TqContractError err{nullptr, 0};
    int32_t r;
    if (w.prefill) {
      std::vector<uint32_t> qc(w.q_per_seq.begin(), w.q_per_seq.end());
      r = tq_mla_prefill_validate(&s, qc.data(), qc.size(), p, &err);
    } else {
      std::vector<uint8_t> qc(w.q_per_seq.begin(), w.q_per_seq.end());
      r = tq_mla_validate(&s, qc.data(), qc.size(), p, &err);
    }
    if (r != TQ_OK) {
      std::fprintf(stderr, "tq_bench: validation: %s %s\n", err.field ? err.field : "",
                   tq_mla_status_string(r));
      std::exit(1);
    }
  };
  auto launch_fn = w.prefill ? tq_mla_prefill : tq_mla_decode;
  TqMlaParams params;
  make_params(dev, &params);
  uint64_t ws_bytes = 0;
  ckt(tq_mla_workspace_bytes(&params, device, &ws_bytes), "workspace");
  void* ws = nullptr;
  ck(cudaMalloc(&ws, ws_bytes), "workspace");
  auto step = [&]() { ckt(launch_fn(&params, ws, ws_bytes, st, nullptr), "launch"); };

  cudaEvent_t e0, e1;
  ck(cudaEventCreate(&e0), "event");
  ck(cudaEventCreate(&e1), "event");
  auto elapsed = [&](cudaEvent_t a, cudaEvent_t b) {
    float ms = 0;
    ck(cudaEventElapsedTime(&ms, a, b), "elapsed");
    return double(ms);
  };

  for (int i = 0; i < warmup; ++i) step();
  ck(cudaStreamSynchronize(st), "warmup");
  int32_t flags = 0;
  ckt(tq_mla_read_device_error(ws, st, &flags), "flags");
  if (flags) die("device error flag after warm-up", flags);

  // ---- whole timed region: K steps back to back, events only at its ends
  ck(cudaEventRecord(e0, st), "record");
  for (int i = 0; i < steps; ++i) step();
  ck(cudaEventRecord(e1, st), "record");
  ck(cudaEventSynchronize(e1), "sync");
  const double ms_step = elapsed(e0, e1) / steps;

  // ---- the attention kernel alone (events around it; its own pass, right after the timed
  // region so that both see the same clocks)
  const int k_steps = std::min(steps, 300);
  std::vector<cudaEvent_t> kb(k_steps), ke(k_steps);
  for (int i = 0; i < k_steps; ++i) {
    ck(cudaEventCreate(&kb[i]), "event");
    ck(cudaEventCreate(&ke[i]), "event");
  }
  for (int i = 0; i < k_steps; ++i) {
    ckt(tq_mla_set_kernel_timer(kb[i], ke[i]), "timer");
    step();
  }
  ckt(tq_mla_set_kernel_timer(nullptr, nullptr), "timer");
  ck(cudaStreamSynchronize(st), "sync");
  double kernel_ms = 0;
  for (int i = 0; i < k_steps; ++i) kernel_ms += elapsed(kb[i], ke[i]);
  kernel_ms /= k_steps;

  // ---- timed runs: R runs of S steps, events at run boundaries only
  std::vector<cudaEvent_t> rev(runs + 1);
  for (auto& e : rev) ck(cudaEventCreate(&e), "event");
  ck(cudaEventRecord(rev[0], st), "record");
  for (int r = 0; r < runs; ++r) {
    for (int i = 0; i < per_run; ++i) step();
    ck(cudaEventRecord(rev[r + 1], st), "record");
  }
  ck(cudaStreamSynchronize(st), "sync");
  std::vector<double> per_step;
  for (int r = 0; r < runs; ++r) per_step.push_back(elapsed(rev[r], rev[r + 1]) / per_run);
  const Stats rs = stats_of(per_step);

  // ---- graph replay: S steps captured once, replayed per run
  Stats gs{};
  if (graph) {
    cudaGraph_t g;
    cudaGraphExec_t ge;
    ck(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "capture");
    for (int i = 0; i < per_run; ++i) step();
    ck(cudaStreamEndCapture(st, &g), "capture");
    ck(cudaGraphInstantiate(&ge, g, 0), "instantiate");
    ck(cudaGraphLaunch(ge, st), "replay");
    ck(cudaEventRecord(rev[0], st), "record");
    for (int r = 0; r < runs; ++r) {
      ck(cudaGraphLaunch(ge, st), "replay");
      ck(cudaEventRecord(rev[r + 1], st), "record");
    }
    ck(cudaStreamSynchronize(st), "sync");
    std::vector<double> g_step;
    for (int r = 0; r < runs; ++r) g_step.push_back(elapsed(rev[r], rev[r + 1]) / per_run);
    gs = stats_of(g_step);
    ck(cudaGraphExecDestroy(ge), "graph");
    ck(cudaGraphDestroy(g), "graph");
  }

  // ---- end to end: inputs from pinned host memory, results back, two buffer sets pipelined
  // over copy-in, compute and copy-out streams (step k+1's copies in and step k-1's copies out
  // overlap step k's compute; every step's own copies stay inside the timed region).
  void *h_q = nullptr, *h_meta = nullptr;
  ck(cudaMallocHost(&h_q, dev.q_bytes), "pinned");
  ck(cudaMallocHost(&h_meta, dev.meta_bytes), "pinned");
  ck(cudaMemcpy(h_q, dev.q, dev.q_bytes, cudaMemcpyDeviceToHost), "q");
  std::memcpy(h_meta, h_meta_buf.data(), dev.meta_bytes);
  struct Set {
    Device d;
    TqMlaParams p;
    void* ws;
    void *h_out, *h_lse;
    cudaEvent_t in, done, out;
  } sets[2];
  for (auto& s : sets) {
    alloc_set(s.d, false, &dev);
    make_params(s.d, &s.p);
    ck(cudaMalloc(&s.ws, ws_bytes), "workspace");
    ck(cudaMallocHost(&s.h_out, s.d.out_bytes), "pinned");
    ck(cudaMallocHost(&s.h_lse, s.d.lse_bytes), "pinned");
    ck(cudaEventCreateWithFlags(&s.in, cudaEventDisableTiming), "event");
    ck(cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming), "event");
    ck(cudaEventCreateWithFlags(&s.out, cudaEventDisableTiming), "event");
    ck(cudaEventRecord(s.done, st), "record");
    ck(cudaEventRecord(s.out, st), "record");
  }
  auto e2e_step = [&](int i) {
    Set& s = sets[i & 1];
    ck(cudaStreamWaitEvent(s_in, s.done, 0), "wait");
    ck(cudaMemcpyAsync(s.d.q, h_q, s.d.q_bytes, cudaMemcpyHostToDevice, s_in), "h2d");
    ck(cudaMemcpyAsync(s.d.meta, h_meta, s.d.meta_bytes, cudaMemcpyHostToDevice, s_in), "h2d");
    ck(cudaEventRecord(s.in, s_in), "record");
    ck(cudaStreamWaitEvent(st, s.in, 0), "wait");
    ck(cudaStreamWaitEvent(st, s.out, 0), "wait");
    ckt(launch_fn(&s.p, s.ws, ws_bytes, st, nullptr), "launch");
    ck(cudaEventRecord(s.done, st), "record");
    ck(cudaStreamWaitEvent(s_out, s.done, 0), "wait");
    ck(cudaMemcpyAsync(s.h_out, s.d.out, s.d.out_bytes, cudaMemcpyDeviceToHost, s_out), "d2h");
    ck(cudaMemcpyAsync(s.h_lse, s.d.lse, s.d.lse_bytes, cudaMemcpyDeviceToHost, s_out), "d2h");
    ck(cudaEventRecord(s.out, s_out), "record");
  };
  for (int i = 0; i < std::max(2, warmup); ++i) e2e_step(i);
  ck(cudaDeviceSynchronize(), "sync");
  ck(cudaEventRecord(e0, st), "record");
  ck(cudaStreamWaitEvent(s_in, e0, 0), "wait");
  ck(cudaStreamWaitEvent(s_out, e0, 0), "wait");
  for (int i = 0; i < steps; ++i) e2e_step(i);
  cudaEvent_t j_in, j_out;
  ck(cudaEventCreateWithFlags(&j_in, cudaEventDisableTiming), "event");
  ck(cudaEventCreateWithFlags(&j_out, cudaEventDisableTiming), "event");
  ck(cudaEventRecord(j_in, s_in), "record");
  ck(cudaEventRecord(j_out, s_out), "record");
  ck(cudaStreamWaitEvent(st, j_in, 0), "wait");
  ck(cudaStreamWaitEvent(st, j_out, 0), "wait");
  ck(cudaEventRecord(e1, st), "record");
  ck(cudaDeviceSynchronize(), "sync");
  const double e2e_ms = elapsed(e0, e1) / steps;
  // The end-to-end results equal the resident run's bit for bit (same inputs, deterministic).
  std::vector<uint8_t> r_out(dev.out_bytes), r_lse(dev.lse_bytes);
  step();
  ck(cudaMemcpy(r_out.data(), dev.out, dev.out_bytes, cudaMemcpyDeviceToHost), "out");
  ck(cudaMemcpy(r_lse.data(), dev.lse, dev.lse_bytes, cudaMemcpyDeviceToHost), "lse");
  bool same = true;
  for (auto& s : sets)
    same = same && !std::memcmp(s.h_out, r_out.data(), dev.out_bytes) &&
           !std::memcmp(s.h_lse, r_lse.data(), dev.lse_bytes);
  int32_t flags_all = 0;
  for (auto& s : sets) {
    ckt(tq_mla_read_device_error(s.ws, st, &flags), "flags");
    flags_all |= flags;
  }
  ckt(tq_mla_read_device_error(ws, st, &flags), "flags");
  flags_all |= flags;
  if (!dump_out.empty()) {
    FILE* f = std::fopen(dump_out.c_str(), "wb");
    if (!f) die("cannot open --dump-out", 0);
    const bool ok = std::fwrite(r_out.data(), 1, r_out.size(), f) == r_out.size() &&
                    std::fwrite(r_lse.data(), 1, r_lse.size(), f) == r_lse.size();
    std::fclose(f);
    if (!ok) die("short write to --dump-out", 0);
  }

  const double tokens = double(T);
  const uint64_t h2d = dev.q_bytes + dev.meta_bytes, d2h = dev.out_bytes + dev.lse_bytes;
  std::printf(
      "{\"impl\": \"native\", \"binary\": \"tq_bench\", \"metric\": \"MLA paged decode tokens/s\", "
      "\"unit\": \"tokens/s\", \"workload\": \"%s\", \"world\": %d, \"rank\": %d, "
      "\"tokens\": %lld, \"sequences\": %lld, \"steps\": %d, \"warmup\": %d, "
      "\"ms_per_step\": %.9g, \"value\": %.9g, "
      "\"step_stats\": {\"runs\": %d, \"steps_per_run\": %d, \"ms_p10\": %.9g, "
      "\"ms_median\": %.9g, \"ms_p90\": %.9g, \"ms_iqr\": %.9g, \"ms_mean\": %.9g}, ",
      w.name.c_str(), world, rank, (long long)T, (long long)S, steps, warmup, ms_step,
      tokens / (ms_step * 1e-3), runs, per_run, rs.p10, rs.median, rs.p90, rs.p75 - rs.p25,
      rs.mean);
  if (graph)
    std::printf(
        "\"graph_stats\": {\"runs\": %d, \"steps_per_graph\": %d, \"ms_p10\": %.9g, "
        "\"ms_median\": %.9g, \"ms_p90\": %.9g, \"ms_iqr\": %.9g, \"ms_mean\": %.9g}, ",
        runs, per_run, gs.p10, gs.median, gs.p90, gs.p75 - gs.p25, gs.mean);
  std::printf(
      "\"kernel_ms_per_launch\": %.9g, \"algorithmic_bytes_per_launch\": %.17g, "
      "\"flops_per_launch\": %.17g, "
      "\"e2e\": {\"value\": %.9g, \"unit\": \"tokens/s\", \"h2d_bytes_per_step\": %llu, "
      "\"d2h_bytes_per_step\": %llu, \"ms_per_step\": %.9g, \"results_equal_resident_run\": %s, "
      "\"pipeline\": \"copy-in, compute and copy-out streams, two buffer sets\"}, "
      "\"gpu_launches\": %d, \"device_error_flags\": %d, \"launches_per_step\": %d}\n",
      kernel_ms, w.bytes(), w.flops(), tokens / (e2e_ms * 1e-3), (unsigned long long)h2d,
      (unsigned long long)d2h, e2e_ms, same ? "true" : "false", 3 * steps, flags_all, 3);
  return flags_all == 0 && same ? 0 : 2;
}
