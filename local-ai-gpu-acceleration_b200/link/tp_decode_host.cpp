// tp_decode_host.cpp -- a native host runner of the tensor-parallel decode step, built
// the way the reference builds its apps: the reference's own runtime core decides
// admission and owns device memory, libqgemv_b200.so does the step.
//
// One process per GPU (rank R of N).  Per rank:
//  1. Estimate this rank's device memory: its weight shards, its KV-cache heads, the
//     decoder workspace (qg_decoder_workspace_bytes), the exchange region
//     (qg_decoder_exchange_bytes) and one CUDA graph per context bucket
//     (rtxllm::build_cuda_graph_bucket_plan, runtime/core/graphs/cuda_graph_bucket.h:119-139).
//  2. rtxllm::decide_admission(Strict, {free VRAM, guard}, estimate)
//     (runtime/core/scheduler/admission.cpp:68-99).  The ranks agree through files in the
//     rendezvous directory: if any rank is rejected, every rank prints the bench-contract
//     rejection object and exits 2 (runtime/apps/mixed_sequence_benchmark_runner/main.cpp:3741-3761).
//  3. rtxllm::VramSuperallocator arenas (runtime/core/allocator/vram_superallocator.h:36-44)
//     for weights, KV cache, workspace, exchange and I/O; seeded synthetic weights (every rank
//     draws the same global tensors and keeps its shards) copied in; the decoder created in
//     the arenas (qg_decoder_create_in: the library allocates nothing).
//  4. One graph per context bucket (rtxllm::CudaGraphBucket), captured around
//     qg_decoder_step_at with the position in device memory and advanced on the device;
//     tokens 0 .. T-1 replay the smallest bucket that covers their position.  The same
//     tokens are also run eagerly (qg_decoder_step, host positions) on a second copy of
//     the KV cache, and the runner reports whether the graphs reproduced them bit for bit.
// Output: one JSON object on stdout; exit 0 (ran), 2 (admission rejected), 1 (error).
#include <cuda_runtime_api.h>

#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <iostream>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "include/qgemv_b200.h"
#include "runtime/core/allocator/vram_superallocator.h"
#include "runtime/core/graphs/cuda_graph_bucket.h"
#include "runtime/core/scheduler/admission.h"

namespace {

struct Options {
  uint32_t tp = 1, rank = 0;
  std::filesystem::path rendezvous;
  uint32_t layers = 80, hidden = 8192, n_q = 64, n_kv = 8, ffn = 28672, vocab = 128256;
  uint32_t ctx_max = 4096;
  std::vector<uint32_t> buckets = {512, 1024, 2048, 4096};
  uint32_t tokens = 8;
  uint64_t vram_free_override = 0;  // testing: the free-VRAM figure admission sees
  uint64_t guard_mib = 512;
  bool admission_only = false;
  uint64_t seed = 1;
};

[[noreturn]] void usage_error(const std::string& msg) { throw std::invalid_argument(msg); }

std::vector<uint32_t> parse_list(const std::string& s) {
  std::vector<uint32_t> out;
  std::stringstream ss(s);
  std::string item;
  while (std::getline(ss, item, ',')) out.push_back(static_cast<uint32_t>(std::stoul(item)));
  return out;
}

Options parse(int argc, char** argv) {
  Options o;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto val = [&]() -> std::string {
      if (i + 1 >= argc) usage_error(a + " needs a value");
      return argv[++i];
    };
    if (a == "--tp") o.tp = std::stoul(val());
    else if (a == "--rank") o.rank = std::stoul(val());
    else if (a == "--rendezvous") o.rendezvous = val();
    else if (a == "--layers") o.layers = std::stoul(val());
    else if (a == "--hidden") o.hidden = std::stoul(val());
    else if (a == "--q-heads") o.n_q = std::stoul(val());
    else if (a == "--kv-heads") o.n_kv = std::stoul(val());
    else if (a == "--ffn") o.ffn = std::stoul(val());
    else if (a == "--vocab") o.vocab = std::stoul(val());
    else if (a == "--ctx-max") o.ctx_max = std::stoul(val());
    else if (a == "--ctx-buckets") o.buckets = parse_list(val());
    else if (a == "--tokens") o.tokens = std::stoul(val());
    else if (a == "--vram-free-bytes") o.vram_free_override = std::stoull(val());
    else if (a == "--guard-mib") o.guard_mib = std::stoull(val());
    else if (a == "--admission-only") o.admission_only = true;
    else if (a == "--seed") o.seed = std::stoull(val());
    else usage_error("unknown argument: " + a);
  }
  if (o.tp == 0 || o.rank >= o.tp) usage_error("--rank must be below --tp");
  if (o.tp > 1 && o.rendezvous.empty()) usage_error("--rendezvous DIR is required with --tp > 1");
  std::sort(o.buckets.begin(), o.buckets.end());
  if (o.buckets.empty() || o.buckets.back() > o.ctx_max) usage_error("buckets must be <= --ctx-max");
  return o;
}

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
  }
}

size_t align256(size_t v) { return (v + 255u) & ~size_t(255); }

// Counter-based generator (splitmix64): every rank draws identical global tensors.
struct Rng {
  uint64_t s;
  uint64_t next() {
    uint64_t z = (s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  float uniform() { return static_cast<float>((next() >> 40) * (1.0 / 16777216.0)); }
  float normal() {  // sum of 12 uniforms, mean 0, variance 1
    float a = 0.f;
    for (int i = 0; i < 12; ++i) a += uniform();
    return a - 6.0f;
  }
};

uint16_t f32_to_f16(float f) {  // round to nearest even, finite normal range only
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  int32_t exp = static_cast<int32_t>((x >> 23) & 0xffu) - 127 + 15;
  uint32_t mant = x & 0x7fffffu;
  if (exp <= 0) return static_cast<uint16_t>(sign);  // flush the (unused) subnormal range
  if (exp >= 31) return static_cast<uint16_t>(sign | 0x7c00u);
  uint32_t h = sign | (static_cast<uint32_t>(exp) << 10) | (mant >> 13);
  const uint32_t rest = mant & 0x1fffu;
  if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) ++h;
  return static_cast<uint16_t>(h);
}

// A pack of the BASELINE distributions: every byte uniform, fp16 d (and dmin) in [1e-3, 1e-2].
std::vector<uint8_t> synthetic_pack(int fmt, uint32_t rows, uint32_t cols, Rng& rng) {
  const uint32_t bb = qg_payload_bytes_per_block(fmt);
  const size_t nblocks = static_cast<size_t>(rows) * (cols / 256u);
  std::vector<uint8_t> p(nblocks * bb);
  for (size_t i = 0; i < p.size(); i += 8) {
    const uint64_t v = rng.next();
    std::memcpy(p.data() + i, &v, std::min<size_t>(8, p.size() - i));
  }
  const int nscale = (fmt == QG_FMT_Q4K_RAW || fmt == QG_FMT_Q5K) ? 2 : 1;
  for (size_t b = 0; b < nblocks; ++b) {
    for (int k = 0; k < nscale; ++k) {
      const uint16_t h = f32_to_f16(1e-3f + 9e-3f * rng.uniform());
      std::memcpy(p.data() + b * bb + 2 * k, &h, 2);
    }
  }
  return p;
}

std::vector<uint8_t> rows_of(const std::vector<uint8_t>& full, int fmt, uint32_t cols, uint32_t r0,
                             uint32_t r1) {
  const size_t row = static_cast<size_t>(cols / 256u) * qg_payload_bytes_per_block(fmt);
  return std::vector<uint8_t>(full.begin() + r0 * row, full.begin() + r1 * row);
}

std::vector<uint8_t> cols_of(const std::vector<uint8_t>& full, int fmt, uint32_t rows, uint32_t cols,
                             uint32_t c0, uint32_t c1) {
  const size_t bb = qg_payload_bytes_per_block(fmt), bpr = cols / 256u;
  const size_t b0 = c0 / 256u, nb = (c1 - c0) / 256u;
  std::vector<uint8_t> out(static_cast<size_t>(rows) * nb * bb);
  for (uint32_t r = 0; r < rows; ++r) {
    std::memcpy(out.data() + r * nb * bb, full.data() + (r * bpr + b0) * bb, nb * bb);
  }
  return out;
}

void write_file(const std::filesystem::path& p, const std::string& text) {
  const auto tmp = p.string() + ".tmp";
  {
    std::ofstream f(tmp, std::ios::binary);
    f << text;
  }
  std::filesystem::rename(tmp, p);
}

std::string read_file_wait(const std::filesystem::path& p, double seconds) {
  const auto until = std::chrono::steady_clock::now() + std::chrono::duration<double>(seconds);
  while (std::chrono::steady_clock::now() < until) {
    std::ifstream f(p, std::ios::binary);
    if (f) {
      std::stringstream ss;
      ss << f.rdbuf();
      return ss.str();
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(20));
  }
  throw std::runtime_error("rendezvous timed out waiting for " + p.string());
}

void print_rejection(const Options& o, const rtxllm::AdmissionDecision& mine, uint32_t rejected_rank,
                     const std::string& reason) {
  const auto& b = mine.breakdown;
  std::cout << "{\n  \"path\": \"tp_decode_host\",\n  \"admitted\": false,\n"
            << "  \"rank\": " << o.rank << ",\n  \"tp\": " << o.tp << ",\n"
            << "  \"rejected_rank\": " << rejected_rank << ",\n"
            << "  \"reason\": \"" << reason << "\",\n"
            << "  \"required_bytes\": " << b.required_bytes << ",\n"
            << "  \"usable_bytes\": " << b.usable_bytes << ",\n"
            << "  \"over_budget_bytes\": " << b.over_budget_bytes << ",\n"
            << "  \"weight_bytes\": " << b.weight_bytes << ",\n"
            << "  \"kv_cache_bytes\": " << b.kv_cache_bytes << ",\n"
            << "  \"workspace_bytes\": " << b.workspace_bytes << ",\n"
            << "  \"graph_bytes\": " << b.graph_bytes << "\n}\n";
}

int run(const Options& o) {
  qg_decoder_dims d{};
  d.layers = o.layers;
  d.hidden = o.hidden;
  d.n_q_heads = o.n_q;
  d.n_kv_heads = o.n_kv;
  d.head_dim = 128;
  d.ffn = o.ffn;
  d.vocab = o.vocab;
  d.ctx_max = o.ctx_max;
  d.eps = 1e-5f;
  d.rope_base = 500000.0f;
  d.attn_fmt = QG_FMT_IQ3S;
  d.ffn_fmt = QG_FMT_IQ2S;
  d.down_fmt = QG_FMT_Q5K;
  d.head_fmt = QG_FMT_Q4K_RAW;
  d.tp_rank = o.rank;
  d.tp_size = o.tp;
  d.collective = 0;
  uint32_t q_rows = 0, kv_rows = 0, ffn_rows = 0, vocab_rows = 0, vocab_off = 0;
  check(qg_decoder_shard(&d, &q_rows, &kv_rows, &ffn_rows, &vocab_rows, &vocab_off), "qg_decoder_shard");
  size_t ws_bytes = 0, ex_bytes = 0;
  check(qg_decoder_workspace_bytes(&d, &ws_bytes), "qg_decoder_workspace_bytes");
  check(qg_decoder_exchange_bytes(&d, &ex_bytes), "qg_decoder_exchange_bytes");

  // 1. this rank's estimate
  auto pb = [](int fmt, uint32_t r, uint32_t c) {
    return align256(static_cast<size_t>(r) * (c / 256u) * qg_payload_bytes_per_block(fmt));
  };
  size_t weight_bytes = 0;
  for (uint32_t l = 0; l < o.layers; ++l) {
    weight_bytes += 2 * align256(4ull * o.hidden);
    weight_bytes += pb(d.attn_fmt, q_rows, o.hidden) + 2 * pb(d.attn_fmt, kv_rows, o.hidden) +
                    pb(d.attn_fmt, o.hidden, q_rows) + 2 * pb(d.ffn_fmt, ffn_rows, o.hidden) +
                    pb(d.down_fmt, o.hidden, ffn_rows);
  }
  weight_bytes += align256(4ull * o.hidden) + pb(d.head_fmt, vocab_rows, o.hidden);
  const size_t kv_layer = align256(2ull * (kv_rows / 128u) * o.ctx_max * 128u);  // fp16
  const size_t kv_bytes = 2ull * o.layers * kv_layer;                          // K and V
  const size_t io_bytes = align256(4ull * o.hidden) + 256;  // x, then token, check token, position
  std::vector<rtxllm::CudaGraphBucketDescriptor> descs;
  for (const uint32_t c : o.buckets) {
    rtxllm::CudaGraphBucketDescriptor g;
    g.name = "decode_ctx" + std::to_string(c);
    g.batch_bucket = 1;
    g.query_bucket = 1;
    g.phase_count = 2 * o.layers + 1;                 // attention + FFN per layer, the head
    g.kernel_launches_per_replay = 10 * o.layers + 4;
    g.workspace_high_water_bytes = ws_bytes;
    descs.push_back(g);
  }
  const auto plan = rtxllm::build_cuda_graph_bucket_plan(descs);
  rtxllm::RequestEstimate est;
  est.weight_bytes = weight_bytes;
  est.prompt_tokens = 0;
  est.max_new_tokens = o.tokens;
  est.kv_bytes_per_token = 0;  // the cache is preallocated for ctx_max positions
  est.kv_cache_bytes = 2 * kv_bytes;  // graph copy + eager check copy
  est.workspace_bytes = 2 * ws_bytes + ex_bytes + io_bytes;
  est.workspace_high_water_bytes = ws_bytes;
  est.graph_bytes = plan.total_bytes;

  // 2. admission, agreed by every rank
  size_t free_bytes = o.vram_free_override;
  if (free_bytes == 0) {
    check(cudaSetDevice(static_cast<int>(o.rank)), "cudaSetDevice");
    size_t total = 0;
    check(cudaMemGetInfo(&free_bytes, &total), "cudaMemGetInfo");
  }
  const auto decision = rtxllm::decide_admission(
      rtxllm::ResidencyPolicy::Strict, rtxllm::MemoryBudget{free_bytes, o.guard_mib << 20}, est);
  uint32_t rejected_rank = decision.admit ? UINT32_MAX : o.rank;
  if (o.tp > 1) {
    write_file(o.rendezvous / ("admit." + std::to_string(o.rank)), decision.admit ? "1" : "0");
    for (uint32_t r = 0; r < o.tp; ++r) {
      const std::string v = read_file_wait(o.rendezvous / ("admit." + std::to_string(r)), 120.0);
      if (v != "1" && rejected_rank == UINT32_MAX) rejected_rank = r;
    }
  }
  if (rejected_rank != UINT32_MAX) {
    print_rejection(o, decision, rejected_rank,
                    rejected_rank == o.rank ? decision.reason : "another rank was rejected");
    return 2;
  }
  if (o.admission_only) {
    std::cout << "{\n  \"path\": \"tp_decode_host\",\n  \"admitted\": true,\n  \"rank\": " << o.rank
              << ",\n  \"required_bytes\": " << decision.required_bytes << ",\n  \"usable_bytes\": "
              << decision.usable_bytes << "\n}\n";
    return 0;
  }

  // 3. arenas and weights
  check(cudaSetDevice(static_cast<int>(o.rank)), "cudaSetDevice");
  rtxllm::VramSuperallocator pool;
  std::vector<rtxllm::ArenaSpec> specs = {{"weights", weight_bytes}, {"kv", kv_bytes},
                                          {"kv_check", kv_bytes}, {"workspace", ws_bytes},
                                          {"workspace_check", ws_bytes}, {"io", io_bytes}};
  if (ex_bytes > 0) specs.push_back({"exchange", ex_bytes});
  pool.initialize(specs);
  uint8_t* wbase = static_cast<uint8_t*>(pool.arena_ptr("weights"));
  size_t woff = 0;
  auto put = [&](const void* src, size_t n) -> uint8_t* {
    uint8_t* dst = wbase + woff;
    check(cudaMemcpy(dst, src, n, cudaMemcpyHostToDevice), "weights upload");
    woff += align256(n);
    return dst;
  };
  Rng rng{o.seed * 0x51ED2701ull + 3};
  const uint32_t q0 = o.rank * q_rows, k0 = o.rank * kv_rows, f0 = o.rank * ffn_rows;
  const uint32_t h0 = o.rank * (o.n_kv / o.tp), nkv_local = o.n_kv / o.tp;
  std::vector<qg_decoder_layer> layers(o.layers);
  uint8_t* kv = static_cast<uint8_t*>(pool.arena_ptr("kv"));
  uint8_t* kv2 = static_cast<uint8_t*>(pool.arena_ptr("kv_check"));
  std::vector<uint16_t> cache_full(static_cast<size_t>(o.n_kv) * o.ctx_max * 128u);
  for (uint32_t l = 0; l < o.layers; ++l) {
    qg_decoder_layer& L = layers[l];
    std::vector<float> an(o.hidden), fn(o.hidden);
    for (auto& v : an) v = 1.0f + 0.02f * rng.normal();
    for (auto& v : fn) v = 1.0f + 0.02f * rng.normal();
    L.attn_norm = reinterpret_cast<const float*>(put(an.data(), 4ull * o.hidden));
    L.ffn_norm = reinterpret_cast<const float*>(put(fn.data(), 4ull * o.hidden));
    const auto wq = synthetic_pack(d.attn_fmt, o.n_q * 128u, o.hidden, rng);
    const auto wk = synthetic_pack(d.attn_fmt, o.n_kv * 128u, o.hidden, rng);
    const auto wv = synthetic_pack(d.attn_fmt, o.n_kv * 128u, o.hidden, rng);
    const auto wo = synthetic_pack(d.attn_fmt, o.hidden, o.n_q * 128u, rng);
    const auto wg = synthetic_pack(d.ffn_fmt, o.ffn, o.hidden, rng);
    const auto wu = synthetic_pack(d.ffn_fmt, o.ffn, o.hidden, rng);
    const auto wd = synthetic_pack(d.down_fmt, o.hidden, o.ffn, rng);
    auto up = [&](const std::vector<uint8_t>& v) { return put(v.data(), v.size()); };
    L.wq = up(rows_of(wq, d.attn_fmt, o.hidden, q0, q0 + q_rows));
    L.wk = up(rows_of(wk, d.attn_fmt, o.hidden, k0, k0 + kv_rows));
    L.wv = up(rows_of(wv, d.attn_fmt, o.hidden, k0, k0 + kv_rows));
    L.wo = up(cols_of(wo, d.attn_fmt, o.hidden, o.n_q * 128u, q0, q0 + q_rows));
    L.wg = up(rows_of(wg, d.ffn_fmt, o.hidden, f0, f0 + ffn_rows));
    L.wu = up(rows_of(wu, d.ffn_fmt, o.hidden, f0, f0 + ffn_rows));
    L.wd = up(cols_of(wd, d.down_fmt, o.hidden, o.ffn, f0, f0 + ffn_rows));
    for (int kvi = 0; kvi < 2; ++kvi) {
      for (auto& v : cache_full) v = f32_to_f16(rng.normal());
      const size_t per_head = static_cast<size_t>(o.ctx_max) * 128u;
      const size_t off = (2ull * l + kvi) * kv_layer;
      for (uint8_t* base : {kv, kv2}) {
        check(cudaMemcpy(base + off, cache_full.data() + h0 * per_head, 2ull * nkv_local * per_head,
                         cudaMemcpyHostToDevice), "cache upload");
      }
      (kvi == 0 ? L.k_cache : L.v_cache) = kv + off;
    }
  }
  std::vector<float> final_norm(o.hidden);
  for (auto& v : final_norm) v = 1.0f + 0.02f * rng.normal();
  const float* fnorm = reinterpret_cast<const float*>(put(final_norm.data(), 4ull * o.hidden));
  const auto head = synthetic_pack(d.head_fmt, o.vocab, o.hidden, rng);
  const uint8_t* head_dev = put(rows_of(head, d.head_fmt, o.hidden, vocab_off, vocab_off + vocab_rows).data(),
                                pb(d.head_fmt, vocab_rows, o.hidden));
  // the eager check decoder reads the second cache copy
  std::vector<qg_decoder_layer> layers2 = layers;
  for (uint32_t l = 0; l < o.layers; ++l) {
    layers2[l].k_cache = kv2 + (2ull * l) * kv_layer;
    layers2[l].v_cache = kv2 + (2ull * l + 1) * kv_layer;
  }

  // NCCL id through the rendezvous directory
  std::vector<uint8_t> id(128, 0);
  if (o.tp > 1) {
    if (o.rank == 0) {
      check(qg_nccl_unique_id(id.data()), "qg_nccl_unique_id");
      write_file(o.rendezvous / "nccl_id", std::string(id.begin(), id.end()));
    } else {
      const std::string v = read_file_wait(o.rendezvous / "nccl_id", 120.0);
      std::memcpy(id.data(), v.data(), std::min<size_t>(128, v.size()));
    }
  }
  uint8_t* io = static_cast<uint8_t*>(pool.arena_ptr("io"));
  float* x = reinterpret_cast<float*>(io);                       // hidden floats
  uint32_t* token = reinterpret_cast<uint32_t*>(io + align256(4ull * o.hidden));
  uint32_t* token2 = token + 1;
  uint32_t* pos = token + 2;
  std::vector<float> xh(o.hidden);
  Rng xr{o.seed * 77 + 5};
  for (auto& v : xh) v = xr.normal();
  check(cudaMemcpy(x, xh.data(), 4ull * o.hidden, cudaMemcpyHostToDevice), "x upload");
  check(cudaMemset(pos, 0, 4), "pos reset");

  // 4. decoders in the arenas (the check decoder is a single-rank run when tp == 1 only:
  //    a second communicator would need a second id, so with tp > 1 both decoders share
  //    the first's ranks in sequence)
  qg_decoder dec = nullptr;
  check(qg_decoder_create_in(&d, layers.data(), fnorm, head_dev, nullptr, pool.arena_ptr("workspace"),
                             ex_bytes ? pool.arena_ptr("exchange") : nullptr, id.data(), &dec),
        "qg_decoder_create_in");
  cudaStream_t stream = nullptr;
  check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreateWithFlags");
  // one eager step first (kernel attributes are set outside any capture); it writes the
  // same K/V at position 0 that the first replay writes again
  check(qg_decoder_step_at(dec, x, pos, o.buckets.front(), 0u, token, stream), "warm-up step");
  check(cudaStreamSynchronize(stream), "warm-up");
  std::vector<std::unique_ptr<rtxllm::CudaGraphBucket>> graphs;
  for (const uint32_t c : o.buckets) {
    cudaGraph_t g = nullptr;
    check(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "capture");
    const cudaError_t e = qg_decoder_step_at(dec, x, pos, c, 1u, token, stream);
    check(cudaStreamEndCapture(stream, &g), "end capture");
    check(e, "qg_decoder_step_at");
    graphs.push_back(std::make_unique<rtxllm::CudaGraphBucket>());
    graphs.back()->instantiate(g);
  }
  std::vector<uint32_t> graph_tokens, eager_tokens, replays(o.buckets.size(), 0);
  std::vector<double> bucket_ms(o.buckets.size(), 0.0);
  cudaEvent_t e0, e1;
  check(cudaEventCreate(&e0), "event");
  check(cudaEventCreate(&e1), "event");
  for (uint32_t t = 0; t < o.tokens; ++t) {
    const size_t b = std::lower_bound(o.buckets.begin(), o.buckets.end(), t + 1) - o.buckets.begin();
    if (b == o.buckets.size()) throw std::runtime_error("token position past the largest bucket");
    check(cudaEventRecord(e0, stream), "record");
    graphs[b]->replay(stream);
    check(cudaEventRecord(e1, stream), "record");
    check(cudaStreamSynchronize(stream), "replay");
    float ms = 0.f;
    check(cudaEventElapsedTime(&ms, e0, e1), "elapsed");
    bucket_ms[b] += ms;
    ++replays[b];
    uint32_t tok = 0;
    check(cudaMemcpy(&tok, token, 4, cudaMemcpyDeviceToHost), "token");
    graph_tokens.push_back(tok);
  }
  std::vector<float> hidden_graph(o.hidden), hidden_eager(o.hidden);
  float* hview = nullptr;
  check(qg_decoder_views(dec, &hview, nullptr), "views");
  check(cudaMemcpy(hidden_graph.data(), hview, 4ull * o.hidden, cudaMemcpyDeviceToHost), "hidden");
  graphs.clear();
  check(qg_decoder_destroy(dec), "destroy");
  uint32_t errors = 0;
  check(qg_get_error(&errors), "qg_get_error");

  // the same tokens eagerly, host positions, second cache copy (same exchange region and
  // workspace: the first decoder is gone)
  qg_decoder dec2 = nullptr;
  if (o.tp > 1) {  // a fresh communicator needs a fresh id
    const std::string name = "nccl_id2";
    if (o.rank == 0) {
      check(qg_nccl_unique_id(id.data()), "qg_nccl_unique_id");
      write_file(o.rendezvous / name, std::string(id.begin(), id.end()));
    } else {
      const std::string v = read_file_wait(o.rendezvous / name, 120.0);
      std::memcpy(id.data(), v.data(), std::min<size_t>(128, v.size()));
    }
  }
  check(qg_decoder_create_in(&d, layers2.data(), fnorm, head_dev, nullptr,
                             pool.arena_ptr("workspace_check"),
                             ex_bytes ? pool.arena_ptr("exchange") : nullptr, id.data(), &dec2),
        "qg_decoder_create_in (check)");
  for (uint32_t t = 0; t < o.tokens; ++t) {
    check(qg_decoder_step(dec2, x, t, token2, stream), "qg_decoder_step");
    check(cudaStreamSynchronize(stream), "step");
    uint32_t tok = 0;
    check(cudaMemcpy(&tok, token2, 4, cudaMemcpyDeviceToHost), "token");
    eager_tokens.push_back(tok);
  }
  check(qg_decoder_views(dec2, &hview, nullptr), "views");
  check(cudaMemcpy(hidden_eager.data(), hview, 4ull * o.hidden, cudaMemcpyDeviceToHost), "hidden");
  check(qg_decoder_destroy(dec2), "destroy");
  const bool same = graph_tokens == eager_tokens &&
                    std::memcmp(hidden_graph.data(), hidden_eager.data(), 4ull * o.hidden) == 0;
  uint32_t pos_end = 0;
  check(cudaMemcpy(&pos_end, pos, 4, cudaMemcpyDeviceToHost), "pos");

  std::cout << "{\n  \"path\": \"tp_decode_host\",\n  \"admitted\": true,\n"
            << "  \"rank\": " << o.rank << ",\n  \"tp\": " << o.tp << ",\n"
            << "  \"layers\": " << o.layers << ",\n  \"tokens\": " << o.tokens << ",\n"
            << "  \"required_bytes\": " << decision.required_bytes << ",\n"
            << "  \"usable_bytes\": " << decision.usable_bytes << ",\n"
            << "  \"allocated_bytes\": " << pool.total_bytes() << ",\n"
            << "  \"graph_plan_bytes\": " << plan.total_bytes << ",\n  \"buckets\": [";
  for (size_t b = 0; b < o.buckets.size(); ++b) {
    std::cout << (b ? ", " : "") << "{\"ctx\": " << o.buckets[b] << ", \"replays\": " << replays[b]
              << ", \"ms_per_token\": " << (replays[b] ? bucket_ms[b] / replays[b] : 0.0) << "}";
  }
  std::cout << "],\n  \"position_after\": " << pos_end << ",\n  \"tokens_graph\": [";
  for (size_t i = 0; i < graph_tokens.size(); ++i) std::cout << (i ? ", " : "") << graph_tokens[i];
  std::cout << "],\n  \"graph_matches_eager\": " << (same ? "true" : "false") << ",\n"
            << "  \"error_word\": " << errors << "\n}\n";
  check(cudaStreamDestroy(stream), "stream destroy");
  return (same && errors == 0 && pos_end == o.tokens) ? 0 : 3;
}

}  // namespace

int main(int argc, char** argv) {
  try {
    return run(parse(argc, argv));
  } catch (const std::exception& e) {
    std::cerr << "tp_decode_host failed: " << e.what() << "\n";
    return 1;
  }
}
