// qg_decode.cu -- tensor-parallel decode step of a Llama-style mixed-quant model
// host side in C++ with NCCL.
//
// One process per GPU; rank r of N holds:
//   row shards   Wq, Wk, Wv (its n_q/N and n_kv/N heads), Wg, Wu (ffn/N rows),
//                the vocab head (vocab/N rows, remainder to the first ranks);
//   column shards Wo (its q heads' columns), Wd (its ffn/N columns);
//   its kv heads' fp16 KV cache.
// Per layer:  h = rmsnorm(x)*w_attn -> q,k,v (one GEMV launch) -> RoPE + cache append
//   -> GQA decode attention -> Wo (partial) -> exchange -> x1 = x + sum of partials
//   -> rmsnorm*w_ffn -> gate,up (one launch) -> silu(g)*u -> Wd (partial) -> exchange
//   -> x2 = x1 + sum.  After the last layer: final rmsnorm -> vocab-shard GEMV -> shard
//   argmax -> all-gather of (value, index) -> token.
// Every tensor-parallel degree computes the single-GPU step bit for bit: the column-
// parallel rows (Q/K/V, gate/up, head) are whole rows on one rank; the row-parallel
// Wo / Wd sums follow one canonical order (8 column segments = the shards at TP 8,
// each summed in a fixed order, then a pairwise tree; a rank's GEMV computes its
// subtree, the exchange gather adds the ranks in the same tree and then the residual);
// the RMSNorm sum of squares has one fixed order in both the plain and the gathering
// kernel.
// The two exchanges per layer are fused into the kernels around them, over NVLink peer
// memory: the Wo / Wd GEMV stores every output row straight into each rank's exchange
// buffer (this rank's slot) as 64-bit words that carry the exchange's epoch; the next
// kernel (RMSNorm + int8 planes, which reads the whole vector anyway) reads every rank's
// slot until each word is current, sums the ranks and normalises.  No extra launch,
// fence, flag or collective library call on the hot path; buffers are double-buffered
// by epoch parity, so a rank can run at most one exchange ahead of the slowest one.  The
// exchange buffers are allocated by qg_decoder_create and shared through CUDA IPC
// (handles gathered with NCCL once).  NCCL carries only the token's all-gather.  The
// baseline mode (collective = 1) moves the same words with ncclAllGather into a local
// buffer instead of peer stores, so it gives the same bits as well.
// Every launch goes on the caller's stream, so one decode step can be captured into one
// CUDA graph (qg_graph_begin / qg_graph_end).
#include <nccl.h>

#include <cstring>
#include <new>
#include <vector>

#include "qg_host.h"

namespace qg {
// One layer's attention (qg_attn.cu): RoPE, KV append and split in one launch, then the
// combine; `partial` holds attn_partial_floats floats of span records.
cudaError_t attn_partial_floats(uint32_t n_q, uint32_t ctx_max, size_t* floats);
cudaError_t launch_attention(const float* q, const float* k, const float* v, void* k_cache,
                             void* v_cache, uint32_t n_q, uint32_t n_kv, uint32_t ctx_max,
                             uint32_t pos, const uint32_t* pos_dev, uint32_t ctx_limit,
                             float rope_base, float* partial, float* out, void* act,
                             cudaStream_t stream);
cudaError_t launch_argmax_candidate(const float* v, uint32_t n, uint32_t offset, uint32_t* cand,
                                    cudaStream_t stream);
cudaError_t launch_select_token(const uint32_t* cand, uint32_t ranks, uint32_t* token,
                                uint32_t* advance, cudaStream_t stream);
}  // namespace qg

namespace {

constexpr size_t kAlign = 256;
size_t align_up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }

struct Shape {
  uint32_t q_local, kv_local, nq_local, nkv_local, ffn_local, vocab_local, vocab_offset;
};

Shape shard_shape(const qg_decoder_dims* d) {
  Shape s{};
  const uint32_t n = d->tp_size, r = d->tp_rank;
  s.nq_local = d->n_q_heads / n;
  s.nkv_local = d->n_kv_heads / n;
  s.q_local = s.nq_local * d->head_dim;
  s.kv_local = s.nkv_local * d->head_dim;
  s.ffn_local = d->ffn / n;
  const uint32_t base = d->vocab / n, rem = d->vocab % n;
  s.vocab_local = base + (r < rem ? 1u : 0u);
  s.vocab_offset = r * base + (r < rem ? r : rem);
  return s;
}

// Canonical segments of a row-parallel matrix with `full_cols` columns (all ranks): the
// largest P in {8, 4, 2, 1} that cuts the row into whole 256-column blocks; a rank of tp
// holds P / tp of them (tensor-parallel shards are whole blocks, so P >= tp).
qg::GemvCanon canon_of(uint32_t full_cols, uint32_t tp) {
  uint32_t P = 8u;
  while (P > 1u && full_cols % (256u * P) != 0u) P >>= 1;
  qg::GemvCanon c{};
  if (P % tp != 0u) return c;  // no canonical split for this degree (nseg = 0)
  c.nseg = P / tp;
  c.seg_chunks = full_cols / (64u * P);
  return c;
}

bool dims_ok(const qg_decoder_dims* d) {
  if (d == nullptr || d->tp_size == 0u || d->tp_rank >= d->tp_size || d->layers == 0u) return false;
  if (d->head_dim != 128u || d->n_kv_heads == 0u || d->n_q_heads % d->n_kv_heads != 0u) return false;
  if (d->n_q_heads % d->tp_size != 0u || d->n_kv_heads % d->tp_size != 0u) return false;
  const uint32_t group = d->n_q_heads / d->n_kv_heads;
  if (group > 16u || (group & (group - 1u)) != 0u) return false;  // attention: G in {1,2,4,8,16}
  if (d->ffn % d->tp_size != 0u || d->vocab < d->tp_size || d->ctx_max == 0u) return false;
  if (d->collective > 1u || d->tp_size > qg::kMaxExchangeRanks) return false;
  const Shape s = shard_shape(d);
  auto width_ok = [](uint32_t n) { return n != 0u && n % 256u == 0u && n / 64u <= 512u; };
  if (!width_ok(d->hidden) || !width_ok(s.q_local) || !width_ok(s.ffn_local)) return false;
  if (canon_of(d->n_q_heads * d->head_dim, d->tp_size).nseg == 0u ||
      canon_of(d->ffn, d->tp_size).nseg == 0u) {
    return false;
  }
  for (int f : {d->attn_fmt, d->ffn_fmt, d->down_fmt, d->head_fmt}) {
    if (f < 0 || f >= QG_FMT_COUNT) return false;
  }
  return true;
}

struct Layout {
  size_t xa, xb, x1, h, act_x, q, k, v, attn, act_attn, opart, g, u, a, act_a, partial, logits,
      cand, total;
};

Layout layout(const qg_decoder_dims* d) {
  const Shape s = shard_shape(d);
  Layout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes);
    return at;
  };
  size_t partial_floats = 0;
  qg::attn_partial_floats(s.nq_local, d->ctx_max, &partial_floats);
  L.xa = take(4ull * d->hidden);
  L.xb = take(4ull * d->hidden);
  L.x1 = take(4ull * d->hidden);
  L.h = take(4ull * d->hidden);
  L.act_x = take(qg::act_bytes(d->hidden));
  L.q = take(4ull * s.q_local);
  L.k = take(4ull * s.kv_local);
  L.v = take(4ull * s.kv_local);
  L.attn = take(4ull * s.q_local);
  L.act_attn = take(qg::act_bytes(s.q_local));
  L.opart = take(4ull * d->hidden);
  L.g = take(4ull * s.ffn_local);
  L.u = take(4ull * s.ffn_local);
  L.a = take(4ull * s.ffn_local);
  L.act_a = take(qg::act_bytes(s.ffn_local));
  L.partial = take(4ull * partial_floats);
  L.logits = take(4ull * s.vocab_local);
  L.cand = take(8ull * d->tp_size);
  L.total = off;
  return L;
}

cudaError_t nccl_status(ncclResult_t r) {
  return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
}

}  // namespace

// Exchange region of one rank (shared with the peers through CUDA IPC): the local epoch,
// then [2 parities][ranks][hidden] 64-bit words (epoch << 32 | value bits).
constexpr size_t kExHeader = 256;
constexpr size_t kExEpoch = 0;  // byte offset inside the header

size_t exchange_bytes(const qg_decoder_dims& d) {
  return align_up(kExHeader + 2ull * d.tp_size * d.hidden * sizeof(uint64_t));
}

struct qg_decoder_s {
  qg_decoder_dims dims{};
  Shape shape{};
  Layout lay{};
  std::vector<qg_decoder_layer> layers;
  const float* final_norm = nullptr;
  const uint8_t* head = nullptr;
  const uint8_t* head_meta = nullptr;
  uint8_t* ws = nullptr;
  ncclComm_t comm = nullptr;
  uint32_t last_output = 0;  // workspace offset of the last step's final hidden state
  const float* last_input = nullptr;  // the last step's input of its last layer
  uint8_t* ex_local = nullptr;                   // this rank's exchange region
  bool ex_owned = false;                         // allocated here (else caller-owned)
  uint8_t* ex_peer[qg::kMaxExchangeRanks] = {};  // every rank's region (self included)
  void* ex_mapped[qg::kMaxExchangeRanks] = {};   // peers' allocations mapped through IPC
  qg::GemvCanon canon_o{}, canon_d{};            // canonical segments of Wo / Wd on this rank
  bool broken = false;                           // a step failed after enqueueing work
};

namespace {

// Base of the device allocation holding `p` (cuMemGetAddressRange through the runtime's
// driver entry point: the library does not link libcuda itself).
cudaError_t allocation_base(void* p, uint8_t** base) {
  using GetRangeFn = int (*)(unsigned long long* base, size_t* size, unsigned long long ptr);
  static GetRangeFn fn = nullptr;
  if (fn == nullptr) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    const cudaError_t e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q);
    if (e != cudaSuccess) return e;
    if (q != cudaDriverEntryPointSuccess || f == nullptr) return cudaErrorNotSupported;
    fn = reinterpret_cast<GetRangeFn>(f);
  }
  unsigned long long b = 0;
  size_t size = 0;
  if (fn(&b, &size, reinterpret_cast<unsigned long long>(p)) != 0) return cudaErrorInvalidDevicePointer;
  *base = reinterpret_cast<uint8_t*>(b);
  return cudaSuccess;
}

// One rank's record in the IPC all-gather: the handle of the allocation holding its
// exchange region and the region's offset in it.
struct ExchangeRecord {
  cudaIpcMemHandle_t handle;
  uint64_t offset;
  uint8_t pad[128 - sizeof(cudaIpcMemHandle_t) - sizeof(uint64_t)];
};
static_assert(sizeof(ExchangeRecord) == 128, "128-byte records");

// Sets up this rank's exchange region -- `region` (caller-owned, exchange_bytes long) or
// one allocated here -- zeroes it, gathers every rank's IPC record through NCCL (staged in
// the decoder workspace, which no step uses yet) and maps the peers' regions.  The
// all-gather also orders every rank's zeroing of its region before any peer can write
// into it.
cudaError_t exchange_setup(qg_decoder_s* dec, void* region) {
  const uint32_t n = dec->dims.tp_size, r = dec->dims.tp_rank;
  const size_t bytes = exchange_bytes(dec->dims);
  cudaError_t e = cudaSuccess;
  if (region != nullptr) {
    dec->ex_local = static_cast<uint8_t*>(region);
  } else {
    e = cudaMalloc(&dec->ex_local, bytes);
    if (e != cudaSuccess) return e;
    dec->ex_owned = true;
  }
  e = cudaMemset(dec->ex_local, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return e;
  dec->ex_peer[r] = dec->ex_local;
  if (dec->dims.collective != 0u) return cudaSuccess;  // NCCL moves the words: local only
  uint8_t* base = nullptr;
  e = allocation_base(dec->ex_local, &base);
  if (e != cudaSuccess) return e;
  ExchangeRecord mine{};
  e = cudaIpcGetMemHandle(&mine.handle, base);
  if (e != cudaSuccess) return e;
  mine.offset = static_cast<uint64_t>(dec->ex_local - base);
  uint8_t* stage = dec->ws;  // n * 128 bytes of the workspace
  std::vector<ExchangeRecord> all(n);
  e = cudaMemcpy(stage + r * sizeof(mine), &mine, sizeof(mine), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) {
    e = nccl_status(ncclAllGather(stage + r * sizeof(mine), stage, sizeof(mine), ncclUint8, dec->comm,
                                  nullptr));
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(nullptr);
  if (e == cudaSuccess) {
    e = cudaMemcpy(all.data(), stage, n * sizeof(ExchangeRecord), cudaMemcpyDeviceToHost);
  }
  if (e != cudaSuccess) return e;
  for (uint32_t p = 0; p < n; ++p) {
    if (p == r) continue;
    void* ptr = nullptr;
    e = cudaIpcOpenMemHandle(&ptr, all[p].handle, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return e;
    dec->ex_mapped[p] = ptr;
    dec->ex_peer[p] = static_cast<uint8_t*>(ptr) + all[p].offset;
  }
  return cudaSuccess;
}

void exchange_teardown(qg_decoder_s* dec) {
  for (uint32_t p = 0; p < qg::kMaxExchangeRanks; ++p) {
    if (dec->ex_mapped[p] != nullptr) cudaIpcCloseMemHandle(dec->ex_mapped[p]);
    dec->ex_mapped[p] = nullptr;
    dec->ex_peer[p] = nullptr;
  }
  if (dec->ex_owned && dec->ex_local != nullptr) cudaFree(dec->ex_local);
  dec->ex_local = nullptr;
  dec->ex_owned = false;
}

// The Wo / Wd GEMV side of an exchange: this rank's slot in every rank's region (fused
// mode), or in its own region only (NCCL mode: ncclAllGather then copies the slots).
qg::GemvExchange exchange_out(const qg_decoder_s* dec) {
  qg::GemvExchange ex{};
  const uint32_t n = dec->dims.tp_size, r = dec->dims.tp_rank, hid = dec->dims.hidden;
  ex.n = dec->dims.collective == 0u ? n : 1u;
  ex.stride = n * hid;
  for (uint32_t k = 0; k < ex.n; ++k) {
    const uint32_t p = dec->dims.collective == 0u ? k : r;
    ex.out[k] = reinterpret_cast<uint64_t*>(dec->ex_peer[p] + kExHeader) + static_cast<size_t>(r) * hid;
  }
  ex.epoch = reinterpret_cast<const uint32_t*>(dec->ex_local + kExEpoch);
  return ex;
}

}  // namespace

extern "C" {

cudaError_t qg_nccl_unique_id(void* id_out) {
  if (id_out == nullptr) return cudaErrorInvalidValue;
  ncclUniqueId id;
  const ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return cudaErrorUnknown;
  std::memcpy(id_out, &id, sizeof(id));
  return cudaSuccess;
}

cudaError_t qg_decoder_workspace_bytes(const qg_decoder_dims* d, size_t* bytes) {
  if (!dims_ok(d) || bytes == nullptr) return cudaErrorInvalidValue;
  *bytes = layout(d).total;
  return cudaSuccess;
}

cudaError_t qg_decoder_shard(const qg_decoder_dims* d, uint32_t* q_rows, uint32_t* kv_rows,
                             uint32_t* ffn_rows, uint32_t* vocab_rows, uint32_t* vocab_offset) {
  if (!dims_ok(d)) return cudaErrorInvalidValue;
  const Shape s = shard_shape(d);
  if (q_rows) *q_rows = s.q_local;
  if (kv_rows) *kv_rows = s.kv_local;
  if (ffn_rows) *ffn_rows = s.ffn_local;
  if (vocab_rows) *vocab_rows = s.vocab_local;
  if (vocab_offset) *vocab_offset = s.vocab_offset;
  return cudaSuccess;
}

}  // extern "C"

namespace {

cudaError_t decoder_create(const qg_decoder_dims* d, const qg_decoder_layer* layers,
                           const float* final_norm, const uint8_t* head, const uint8_t* head_meta,
                           void* workspace, void* exchange, const void* nccl_id, qg_decoder* out) {
  if (!dims_ok(d) || layers == nullptr || final_norm == nullptr || head == nullptr ||
      workspace == nullptr || out == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0u ||
      (reinterpret_cast<uintptr_t>(exchange) & 255u) != 0u || (d->tp_size > 1u && nccl_id == nullptr)) {
    return cudaErrorInvalidValue;
  }
  *out = nullptr;
  auto* dec = new (std::nothrow) qg_decoder_s();
  if (dec == nullptr) return cudaErrorMemoryAllocation;
  dec->dims = *d;
  dec->shape = shard_shape(d);
  dec->lay = layout(d);
  dec->layers.assign(layers, layers + d->layers);
  dec->final_norm = final_norm;
  dec->head = head;
  dec->head_meta = head_meta;
  dec->ws = static_cast<uint8_t*>(workspace);
  dec->canon_o = canon_of(d->n_q_heads * d->head_dim, d->tp_size);
  dec->canon_d = canon_of(d->ffn, d->tp_size);
  if (d->tp_size > 1u) {
    ncclUniqueId id;
    std::memcpy(&id, nccl_id, sizeof(id));
    const ncclResult_t r = ncclCommInitRank(&dec->comm, static_cast<int>(d->tp_size), id,
                                            static_cast<int>(d->tp_rank));
    if (r != ncclSuccess) {
      delete dec;
      return cudaErrorUnknown;
    }
    const cudaError_t e = exchange_setup(dec, exchange);
    if (e != cudaSuccess) {
      exchange_teardown(dec);
      ncclCommDestroy(dec->comm);
      delete dec;
      return e;
    }
  }
  *out = dec;
  return cudaSuccess;
}

}  // namespace

extern "C" {

cudaError_t qg_decoder_exchange_bytes(const qg_decoder_dims* d, size_t* bytes) {
  if (!dims_ok(d) || bytes == nullptr) return cudaErrorInvalidValue;
  *bytes = d->tp_size > 1u ? exchange_bytes(*d) : 0u;
  return cudaSuccess;
}

cudaError_t qg_decoder_create(const qg_decoder_dims* d, const qg_decoder_layer* layers,
                              const float* final_norm, const uint8_t* head,
                              const uint8_t* head_meta, void* workspace, const void* nccl_id,
                              qg_decoder* out) {
  return decoder_create(d, layers, final_norm, head, head_meta, workspace, nullptr, nccl_id, out);
}

cudaError_t qg_decoder_create_in(const qg_decoder_dims* d, const qg_decoder_layer* layers,
                                 const float* final_norm, const uint8_t* head,
                                 const uint8_t* head_meta, void* workspace, void* exchange,
                                 const void* nccl_id, qg_decoder* out) {
  if (d != nullptr && d->tp_size > 1u && exchange == nullptr) return cudaErrorInvalidValue;
  return decoder_create(d, layers, final_norm, head, head_meta, workspace, exchange, nccl_id, out);
}

cudaError_t qg_decoder_destroy(qg_decoder dec) {
  if (dec == nullptr) return cudaSuccess;
  cudaError_t e = cudaSuccess;
  exchange_teardown(dec);
  if (dec->comm != nullptr) e = nccl_status(ncclCommDestroy(dec->comm));
  delete dec;
  return e;
}

}  // extern "C"

namespace {

// One decode step.  pos_dev == nullptr: the position is `pos` (host value, baked into
// the launches); else *pos_dev is read on the device, ctx_bucket (>= 1) bounds the
// context the attention grid covers, and `advance` != 0 increments *pos_dev after the
// token is chosen.
cudaError_t decoder_step(qg_decoder dec, const float* x, uint32_t pos, uint32_t* pos_dev,
                         uint32_t ctx_bucket, uint32_t advance, uint32_t* token,
                         cudaStream_t stream) {
  if (dec->broken) return cudaErrorIllegalState;
  const qg_decoder_dims& d = dec->dims;
  const Shape& s = dec->shape;
  const Layout& L = dec->lay;
  uint8_t* w = dec->ws;
  auto F = [&](size_t off) { return reinterpret_cast<float*>(w + off); };
  const bool tp = d.tp_size > 1u;
  float* x1 = F(L.x1);
  float* h = F(L.h);
  float* q = F(L.q);
  float* k = F(L.k);
  float* v = F(L.v);
  float* attn = F(L.attn);
  float* opart = F(L.opart);
  float* g = F(L.g);
  float* u = F(L.u);
  float* a = F(L.a);
  cudaError_t e = cudaSuccess;
  // Once work of this step is enqueued, a failure leaves the exchange epochs of the
  // ranks out of step: the decoder refuses further steps.
  bool enqueued = false;
#define QG_TRY(expr)                         \
  do {                                       \
    e = (expr);                              \
    if (e != cudaSuccess) {                  \
      if (enqueued) dec->broken = true;      \
      return e;                              \
    }                                        \
    enqueued = true;                         \
  } while (0)
  const float* cur = x;
  size_t out_off = L.xa;
  // With tensor parallelism each row-parallel GEMV's partial stays in the exchange
  // buffers until the next RMSNorm gathers it (pending); the gather writes
  // residual + sum of the ranks to its x_out.
  bool pending = false;
  const float* pending_residual = nullptr;
  uint32_t exchanges = 0;  // exchanges of this step so far (the parity of the next one)
  const qg::GemvExchange ex = tp ? exchange_out(dec) : qg::GemvExchange{};
  const uint64_t* ex_buf = tp ? reinterpret_cast<const uint64_t*>(dec->ex_local + kExHeader) : nullptr;
  uint32_t* ex_epoch = tp ? reinterpret_cast<uint32_t*>(dec->ex_local + kExEpoch) : nullptr;
  auto norm = [&](const float* src, float* gathered, const float* weight) -> cudaError_t {
    if (pending) {
      pending = false;
      return qg::launch_gather_norm_prepare(ex_buf, ex_epoch, d.tp_size, ex.stride,
                                            pending_residual, weight, d.hidden, d.eps, gathered, h,
                                            w + L.act_x, stream);
    }
    return qg::launch_norm_prepare(src, weight, d.hidden, d.eps, h, w + L.act_x, stream);
  };
  // Row-parallel projection: dst = residual + W in (TP 1), or this rank's partial into
  // the exchange (the gather adds the ranks and the residual).
  auto project_out = [&](int fmt, const uint8_t* wt, const uint8_t* wm, const float* in,
                         const void* act, float* dst, const float* residual, uint32_t cols,
                         const qg::GemvCanon& canon) -> cudaError_t {
    if (!tp) {
      return qg::launch_gemv_canonical(fmt, wt, wm, in, act, dst, residual, d.hidden, cols, canon,
                                       stream);
    }
    pending = true;
    pending_residual = residual;
    // Every step runs an even number of exchanges and the epoch starts at 0, so the
    // k-th exchange of a step (from 0) has epoch parity (k + 1) & 1.
    const uint32_t parity = (exchanges + 1u) & 1u;
    ++exchanges;
    cudaError_t e2 = qg::launch_gemv_exchange(fmt, wt, wm, in, act, opart, nullptr, d.hidden, cols,
                                              ex, canon, stream);
    if (e2 != cudaSuccess || d.collective == 0u) return e2;
    uint64_t* half = reinterpret_cast<uint64_t*>(dec->ex_local + kExHeader) +
                     static_cast<size_t>(parity) * ex.stride;
    return nccl_status(ncclAllGather(half + static_cast<size_t>(d.tp_rank) * d.hidden, half, d.hidden,
                                     ncclUint64, dec->comm, stream));
  };
  for (uint32_t l = 0; l < d.layers; ++l) {
    const qg_decoder_layer& W = dec->layers[l];
    float* x2 = F(out_off);
    // attention block (the previous layer's exchange is gathered into x_in)
    float* x_in = F(out_off == L.xa ? L.xb : L.xa);
    const bool gathered = pending;
    QG_TRY(norm(cur, x_in, W.attn_norm));
    if (gathered) cur = x_in;
    if (l + 1u == d.layers) dec->last_input = cur;
    {
      const uint8_t* p[3] = {W.wq, W.wk, W.wv};
      const uint8_t* m[3] = {W.wq_meta, W.wk_meta, W.wv_meta};
      float* y[3] = {q, k, v};
      const uint32_t r[3] = {s.q_local, s.kv_local, s.kv_local};
      QG_TRY(qg::launch_gemv_multi(d.attn_fmt, 3, p, m, y, r, d.hidden, h, w + L.act_x, stream));
    }
    QG_TRY(qg::launch_attention(q, k, v, W.k_cache, W.v_cache, s.nq_local, s.nkv_local, d.ctx_max,
                                pos, pos_dev, pos_dev ? ctx_bucket : d.ctx_max, d.rope_base,
                                F(L.partial), attn, w + L.act_attn, stream));
    QG_TRY(project_out(d.attn_fmt, W.wo, W.wo_meta, attn, w + L.act_attn, x1, cur, s.q_local,
                       dec->canon_o));
    // feed-forward block (the exchange of Wo is gathered into x1)
    QG_TRY(norm(x1, x1, W.ffn_norm));
    {
      const uint8_t* p[2] = {W.wg, W.wu};
      const uint8_t* m[2] = {W.wg_meta, W.wu_meta};
      float* y[2] = {g, u};
      const uint32_t r[2] = {s.ffn_local, s.ffn_local};
      QG_TRY(qg::launch_gemv_multi(d.ffn_fmt, 2, p, m, y, r, d.hidden, h, w + L.act_x, stream));
    }
    QG_TRY(qg::launch_silu_gate_prepare(g, u, s.ffn_local, a, w + L.act_a, stream));
    QG_TRY(project_out(d.down_fmt, W.wd, W.wd_meta, a, w + L.act_a, x2, x1, s.ffn_local,
                       dec->canon_d));
    cur = x2;
    out_off = (out_off == L.xa) ? L.xb : L.xa;
  }
  // vocab head (with tensor parallelism the final norm gathers the last layer's output
  // into the residual buffer the next layer would have used)
  if (pending) {
    float* xf = F(out_off == L.xa ? L.xb : L.xa);
    QG_TRY(norm(cur, xf, dec->final_norm));
    cur = xf;
  } else {
    QG_TRY(norm(cur, nullptr, dec->final_norm));
  }
  dec->last_output = static_cast<uint32_t>(reinterpret_cast<const uint8_t*>(cur) - w);
  QG_TRY(qg::launch_gemv(d.head_fmt, dec->head, dec->head_meta, h, w + L.act_x, F(L.logits),
                         nullptr, nullptr, nullptr, 0u, 0u, 0u, s.vocab_local, d.hidden, stream));
  uint32_t* cand = reinterpret_cast<uint32_t*>(w + L.cand);
  QG_TRY(qg::launch_argmax_candidate(F(L.logits), s.vocab_local, s.vocab_offset,
                                     cand + 2u * d.tp_rank, stream));
  if (tp) {
    QG_TRY(nccl_status(ncclAllGather(cand + 2u * d.tp_rank, cand, 2, ncclUint32, dec->comm, stream)));
  }
  QG_TRY(qg::launch_select_token(cand, d.tp_size, token, (pos_dev && advance) ? pos_dev : nullptr,
                                 stream));
#undef QG_TRY
  return cudaSuccess;
}

}  // namespace

extern "C" {

cudaError_t qg_decoder_step(qg_decoder dec, const float* x, uint32_t pos, uint32_t* token,
                            cudaStream_t stream) {
  if (dec == nullptr || x == nullptr || token == nullptr || pos >= dec->dims.ctx_max) {
    return cudaErrorInvalidValue;
  }
  return decoder_step(dec, x, pos, nullptr, 0u, 0u, token, stream);
}

cudaError_t qg_decoder_step_at(qg_decoder dec, const float* x, uint32_t* pos_dev,
                               uint32_t ctx_bucket, uint32_t advance, uint32_t* token,
                               cudaStream_t stream) {
  if (dec == nullptr || x == nullptr || token == nullptr || pos_dev == nullptr ||
      ctx_bucket == 0u || ctx_bucket > dec->dims.ctx_max) {
    return cudaErrorInvalidValue;
  }
  return decoder_step(dec, x, 0u, pos_dev, ctx_bucket, advance, token, stream);
}

cudaError_t qg_decoder_views(qg_decoder dec, float** hidden_out, float** logits) {
  if (dec == nullptr) return cudaErrorInvalidValue;
  if (hidden_out) *hidden_out = reinterpret_cast<float*>(dec->ws + dec->last_output);
  if (logits) *logits = reinterpret_cast<float*>(dec->ws + dec->lay.logits);
  return cudaSuccess;
}

cudaError_t qg_decoder_stage_buffers(qg_decoder dec, qg_decoder_stage_views* v) {
  if (dec == nullptr || v == nullptr) return cudaErrorInvalidValue;
  if (dec->last_input == nullptr) return cudaErrorNotReady;  // no step enqueued yet
  auto F = [&](size_t off) { return reinterpret_cast<float*>(dec->ws + off); };
  const Layout& L = dec->lay;
  v->layer_input = const_cast<float*>(dec->last_input);
  v->q = F(L.q);
  v->k = F(L.k);
  v->v = F(L.v);
  v->attn = F(L.attn);
  v->x1 = F(L.x1);
  v->g = F(L.g);
  v->u = F(L.u);
  v->a = F(L.a);
  v->hidden = F(dec->last_output);
  v->logits = F(L.logits);
  return cudaSuccess;
}

}  // extern "C"
