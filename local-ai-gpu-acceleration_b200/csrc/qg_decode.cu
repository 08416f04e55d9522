// qg_decode.cu -- tensor-parallel decode step of a Llama-style mixed-quant model
// host side in C++ with NCCL.
//
// One process per GPU; rank r of N holds:
//   row shards   Wq, Wk, Wv (its n_q/N and n_kv/N heads), Wg, Wu (ffn/N rows),
//                the vocab head (vocab/N rows, remainder to the first ranks);
//   column shards Wo (its q heads' columns), Wd (its ffn/N columns);
//   its kv heads' fp16 KV cache.
// Per layer:  h = rmsnorm(x)*w_attn -> q,k,v (one GEMV launch) -> RoPE + cache append
//   -> GQA decode attention -> Wo (partial; rank 0 adds the residual x) -> all-reduce
//   -> rmsnorm*w_ffn -> gate,up (one launch) -> silu(g)*u -> Wd (partial; rank 0 adds
//   the residual) -> all-reduce.  After the last layer: final rmsnorm -> vocab-shard GEMV
//   -> shard argmax -> all-gather of (value, index) -> token.
// Every launch and collective goes on the caller's stream, so one decode step can be
// captured into one CUDA graph (qg_graph_begin / qg_graph_end).
#include <nccl.h>

#include <cstring>
#include <new>
#include <vector>

#include "qg_host.h"

namespace qg {
cudaError_t attn_partial_floats(uint32_t n_q, uint32_t ctx_max, size_t* floats);
cudaError_t launch_rope_append(float* q, float* k, const float* v, void* k_cache, void* v_cache,
                               uint32_t n_q, uint32_t n_kv, uint32_t ctx_max, uint32_t pos,
                               float rope_base, cudaStream_t stream);
cudaError_t launch_attention(const float* q, const void* k_cache, const void* v_cache,
                             uint32_t n_q, uint32_t n_kv, uint32_t ctx_max, uint32_t ctx_len,
                             float* partial, float* out, void* act, cudaStream_t stream);
cudaError_t launch_argmax_candidate(const float* v, uint32_t n, uint32_t offset, uint32_t* cand,
                                    cudaStream_t stream);
cudaError_t launch_select_token(const uint32_t* cand, uint32_t ranks, uint32_t* token,
                                cudaStream_t stream);
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

bool dims_ok(const qg_decoder_dims* d) {
  if (d == nullptr || d->tp_size == 0u || d->tp_rank >= d->tp_size || d->layers == 0u) return false;
  if (d->head_dim != 128u || d->n_kv_heads == 0u || d->n_q_heads % d->n_kv_heads != 0u) return false;
  if (d->n_q_heads % d->tp_size != 0u || d->n_kv_heads % d->tp_size != 0u) return false;
  if (d->n_q_heads / d->n_kv_heads > 16u) return false;
  if (d->ffn % d->tp_size != 0u || d->vocab < d->tp_size || d->ctx_max == 0u) return false;
  const Shape s = shard_shape(d);
  auto width_ok = [](uint32_t n) { return n != 0u && n % 256u == 0u && n / 64u <= 512u; };
  if (!width_ok(d->hidden) || !width_ok(s.q_local) || !width_ok(s.ffn_local)) return false;
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
};

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

cudaError_t qg_decoder_create(const qg_decoder_dims* d, const qg_decoder_layer* layers,
                              const float* final_norm, const uint8_t* head,
                              const uint8_t* head_meta, void* workspace, const void* nccl_id,
                              qg_decoder* out) {
  if (!dims_ok(d) || layers == nullptr || final_norm == nullptr || head == nullptr ||
      workspace == nullptr || out == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0u ||
      (d->tp_size > 1u && nccl_id == nullptr)) {
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
  if (d->tp_size > 1u) {
    ncclUniqueId id;
    std::memcpy(&id, nccl_id, sizeof(id));
    const ncclResult_t r = ncclCommInitRank(&dec->comm, static_cast<int>(d->tp_size), id,
                                            static_cast<int>(d->tp_rank));
    if (r != ncclSuccess) {
      delete dec;
      return cudaErrorUnknown;
    }
  }
  *out = dec;
  return cudaSuccess;
}

cudaError_t qg_decoder_destroy(qg_decoder dec) {
  if (dec == nullptr) return cudaSuccess;
  cudaError_t e = cudaSuccess;
  if (dec->comm != nullptr) e = nccl_status(ncclCommDestroy(dec->comm));
  delete dec;
  return e;
}

cudaError_t qg_decoder_step(qg_decoder dec, const float* x, uint32_t pos, uint32_t* token,
                            cudaStream_t stream) {
  if (dec == nullptr || x == nullptr || token == nullptr || pos >= dec->dims.ctx_max) {
    return cudaErrorInvalidValue;
  }
  const qg_decoder_dims& d = dec->dims;
  const Shape& s = dec->shape;
  const Layout& L = dec->lay;
  uint8_t* w = dec->ws;
  auto F = [&](size_t off) { return reinterpret_cast<float*>(w + off); };
  const bool tp = d.tp_size > 1u;
  const bool rank0 = d.tp_rank == 0u;
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
#define QG_TRY(expr)            \
  do {                          \
    e = (expr);                 \
    if (e != cudaSuccess) return e; \
  } while (0)
  const float* cur = x;
  size_t out_off = L.xa;
  for (uint32_t l = 0; l < d.layers; ++l) {
    const qg_decoder_layer& W = dec->layers[l];
    float* x2 = F(out_off);
    // attention block
    QG_TRY(qg::launch_norm_prepare(cur, W.attn_norm, d.hidden, d.eps, h, w + L.act_x, stream));
    {
      const uint8_t* p[3] = {W.wq, W.wk, W.wv};
      const uint8_t* m[3] = {W.wq_meta, W.wk_meta, W.wv_meta};
      float* y[3] = {q, k, v};
      const uint32_t r[3] = {s.q_local, s.kv_local, s.kv_local};
      QG_TRY(qg::launch_gemv_multi(d.attn_fmt, 3, p, m, y, r, d.hidden, h, w + L.act_x, stream));
    }
    QG_TRY(qg::launch_rope_append(q, k, v, W.k_cache, W.v_cache, s.nq_local, s.nkv_local,
                                  d.ctx_max, pos, d.rope_base, stream));
    QG_TRY(qg::launch_attention(q, W.k_cache, W.v_cache, s.nq_local, s.nkv_local, d.ctx_max,
                                pos + 1u, F(L.partial), attn, w + L.act_attn, stream));
    QG_TRY(qg::launch_gemv(d.attn_fmt, W.wo, W.wo_meta, attn, w + L.act_attn, tp ? opart : x1,
                           rank0 ? cur : nullptr, nullptr, nullptr, 0u, 0u, 0u, d.hidden,
                           s.q_local, stream));
    if (tp) {
      QG_TRY(nccl_status(ncclAllReduce(opart, x1, d.hidden, ncclFloat, ncclSum, dec->comm, stream)));
    }
    // feed-forward block
    QG_TRY(qg::launch_norm_prepare(x1, W.ffn_norm, d.hidden, d.eps, h, w + L.act_x, stream));
    {
      const uint8_t* p[2] = {W.wg, W.wu};
      const uint8_t* m[2] = {W.wg_meta, W.wu_meta};
      float* y[2] = {g, u};
      const uint32_t r[2] = {s.ffn_local, s.ffn_local};
      QG_TRY(qg::launch_gemv_multi(d.ffn_fmt, 2, p, m, y, r, d.hidden, h, w + L.act_x, stream));
    }
    QG_TRY(qg::launch_silu_gate_prepare(g, u, s.ffn_local, a, w + L.act_a, stream));
    QG_TRY(qg::launch_gemv(d.down_fmt, W.wd, W.wd_meta, a, w + L.act_a, tp ? opart : x2,
                           rank0 ? x1 : nullptr, nullptr, nullptr, 0u, 0u, 0u, d.hidden,
                           s.ffn_local, stream));
    if (tp) {
      QG_TRY(nccl_status(ncclAllReduce(opart, x2, d.hidden, ncclFloat, ncclSum, dec->comm, stream)));
    }
    cur = x2;
    out_off = (out_off == L.xa) ? L.xb : L.xa;
  }
  dec->last_output = static_cast<uint32_t>(reinterpret_cast<const uint8_t*>(cur) - w);
  // vocab head
  QG_TRY(qg::launch_norm_prepare(cur, dec->final_norm, d.hidden, d.eps, h, w + L.act_x, stream));
  QG_TRY(qg::launch_gemv(d.head_fmt, dec->head, dec->head_meta, h, w + L.act_x, F(L.logits),
                         nullptr, nullptr, nullptr, 0u, 0u, 0u, s.vocab_local, d.hidden, stream));
  uint32_t* cand = reinterpret_cast<uint32_t*>(w + L.cand);
  QG_TRY(qg::launch_argmax_candidate(F(L.logits), s.vocab_local, s.vocab_offset,
                                     cand + 2u * d.tp_rank, stream));
  if (tp) {
    QG_TRY(nccl_status(ncclAllGather(cand + 2u * d.tp_rank, cand, 2, ncclUint32, dec->comm, stream)));
  }
  QG_TRY(qg::launch_select_token(cand, d.tp_size, token, stream));
#undef QG_TRY
  return cudaSuccess;
}

cudaError_t qg_decoder_views(qg_decoder dec, float** hidden_out, float** logits) {
  if (dec == nullptr) return cudaErrorInvalidValue;
  if (hidden_out) *hidden_out = reinterpret_cast<float*>(dec->ws + dec->last_output);
  if (logits) *logits = reinterpret_cast<float*>(dec->ws + dec->lay.logits);
  return cudaSuccess;
}

}  // extern "C"
