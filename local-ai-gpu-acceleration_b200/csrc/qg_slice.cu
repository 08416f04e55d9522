// qg_slice.cu -- host-side (C++) decode-step sequencing: the mixed-format layer slice
// and the CUDA-graph capture/replay of a decode step.
//
// The reference sequences its layer slice stage by stage (launch_stage / launch_sequence,
// runtime/apps/mixed_sequence_benchmark_runner/main.cpp:4002-4071,4622-4638) and replays
// it as one captured graph (:4801-4835).  Here a Llama-style slice is eight launches:
//   norm_prepare(x)            h = rmsnorm(x) * w, and h's int8 planes
//   gemv[Q|K|V](h)             one launch over the three attention projections
//   act_prepare(q)             (attention is a passthrough, as in the reference's
//   gemv[O](q)                  default attention phase mode: O consumes q)
//   act_prepare(o)
//   gemv[gate|up](o)           one launch over both FFN input projections
//   silu_gate_prepare(g, u)    a = silu(g) * u, and a's int8 planes
//   gemv[down](a) + x          residual add fused into the GEMV epilogue
// All buffers are caller-owned (one workspace); nothing here allocates device memory.
#include <algorithm>
#include <cstdlib>
#include <new>
#include <vector>

#include "qg_host.h"

namespace {

constexpr size_t kAlign = 256;

size_t align_up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }

// Workspace carve-up, in order; offsets are 256-B aligned.
struct SliceLayout {
  size_t h, q, k, v, o, g, u, a, act_h, act_q, act_o, act_a, total;
};

SliceLayout slice_layout(const qg_layer_slice* s) {
  SliceLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes);
    return at;
  };
  L.h = take(4ull * s->hidden);
  L.q = take(4ull * s->q_rows);
  L.k = take(4ull * s->kv_rows);
  L.v = take(4ull * s->kv_rows);
  L.o = take(4ull * s->hidden);
  L.g = take(4ull * s->ffn);
  L.u = take(4ull * s->ffn);
  L.a = take(4ull * s->ffn);
  L.act_h = take(qg::act_bytes(s->hidden));
  L.act_q = take(qg::act_bytes(s->q_rows));
  L.act_o = take(qg::act_bytes(s->hidden));
  L.act_a = take(qg::act_bytes(s->ffn));
  L.total = off;
  return L;
}

bool dims_ok(const qg_layer_slice* s) {
  auto ok = [](uint32_t n) { return n != 0u && (n % 256u) == 0u && n / 64u <= 512u; };
  auto fmt_ok = [](int f, const uint8_t* const* metas, int n) {
    if (f < 0 || f >= QG_FMT_COUNT) return false;
    if (qg_meta_bytes_per_block(f) == 0u) return true;
    for (int i = 0; i < n; ++i) {
      if (metas[i] == nullptr) return false;
    }
    return true;
  };
  if (s == nullptr || !ok(s->hidden) || !ok(s->q_rows) || !ok(s->ffn) || s->kv_rows == 0u) {
    return false;
  }
  const uint8_t* am[4] = {s->wq_meta, s->wk_meta, s->wv_meta, s->wo_meta};
  const uint8_t* fm[2] = {s->wg_meta, s->wu_meta};
  const uint8_t* dm[1] = {s->wd_meta};
  return s->norm_weight && s->wq && s->wk && s->wv && s->wo && s->wg && s->wu && s->wd &&
         fmt_ok(s->attn_fmt, am, 4) && fmt_ok(s->ffn_fmt, fm, 2) && fmt_ok(s->down_fmt, dm, 1);
}

// Batched slice workspace: every activation for `batch` rows, then the tensor-core GEMM
// workspace the largest of its GEMVs needs at this batch (none below the threshold).
struct BatchedLayout {
  size_t h, q, k, v, o, g, u, a, y, tc, total;
};

BatchedLayout batched_layout(const qg_layer_slice* s, uint32_t batch) {
  BatchedLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes);
    return at;
  };
  const size_t b = batch;
  L.h = take(4ull * b * s->hidden);
  L.q = take(4ull * b * s->q_rows);
  L.k = take(4ull * b * s->kv_rows);
  L.v = take(4ull * b * s->kv_rows);
  L.o = take(4ull * b * s->hidden);
  L.g = take(4ull * b * s->ffn);
  L.u = take(4ull * b * s->ffn);
  L.a = take(4ull * b * s->ffn);
  L.y = take(4ull * b * s->hidden);
  size_t tc = 0;
  auto need = [&](int fmt, uint32_t rows, uint32_t cols) {
    tc = std::max(tc, qg::batched_gemm_ws_bytes(fmt, batch, rows, cols));
  };
  need(s->attn_fmt, s->q_rows, s->hidden);
  need(s->attn_fmt, s->kv_rows, s->hidden);
  need(s->attn_fmt, s->hidden, s->q_rows);
  need(s->ffn_fmt, s->ffn, s->hidden);
  need(s->down_fmt, s->hidden, s->ffn);
  L.tc = take(tc);
  // batch 1 runs the single-vector slice (fused Q/K/V, prepared activations) in the
  // same workspace
  L.total = batch == 1u ? std::max(off, slice_layout(s).total) : off;
  return L;
}

}  // namespace

struct qg_graph_s {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
};

struct qg_slice_buckets_s {
  struct Bucket {
    uint32_t batch = 0;
    float* x = nullptr;
    float* out = nullptr;
    void* ws = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
  };
  qg_layer_slice slice{};
  std::vector<Bucket> buckets;
};

extern "C" {

cudaError_t qg_layer_slice_workspace_bytes(const qg_layer_slice* s, size_t* bytes) {
  if (!dims_ok(s) || bytes == nullptr) return cudaErrorInvalidValue;
  *bytes = slice_layout(s).total;
  return cudaSuccess;
}

cudaError_t qg_layer_slice_buffers(const qg_layer_slice* s, void* workspace,
                                   qg_layer_slice_views* views) {
  if (!dims_ok(s) || workspace == nullptr || views == nullptr) return cudaErrorInvalidValue;
  const SliceLayout L = slice_layout(s);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  views->h = reinterpret_cast<float*>(w + L.h);
  views->q = reinterpret_cast<float*>(w + L.q);
  views->k = reinterpret_cast<float*>(w + L.k);
  views->v = reinterpret_cast<float*>(w + L.v);
  views->o = reinterpret_cast<float*>(w + L.o);
  views->gate = reinterpret_cast<float*>(w + L.g);
  views->up = reinterpret_cast<float*>(w + L.u);
  views->act = reinterpret_cast<float*>(w + L.a);
  return cudaSuccess;
}

cudaError_t qg_layer_slice_forward(const qg_layer_slice* s, const float* x, float* out,
                                   void* workspace, cudaStream_t stream) {
  if (!dims_ok(s) || x == nullptr || out == nullptr || workspace == nullptr ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0u) {
    return cudaErrorInvalidValue;
  }
  const SliceLayout L = slice_layout(s);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  float* h = reinterpret_cast<float*>(w + L.h);
  float* q = reinterpret_cast<float*>(w + L.q);
  float* k = reinterpret_cast<float*>(w + L.k);
  float* v = reinterpret_cast<float*>(w + L.v);
  float* o = reinterpret_cast<float*>(w + L.o);
  float* g = reinterpret_cast<float*>(w + L.g);
  float* u = reinterpret_cast<float*>(w + L.u);
  float* a = reinterpret_cast<float*>(w + L.a);
  cudaError_t e = qg::launch_norm_prepare(x, s->norm_weight, s->hidden, s->eps, h, w + L.act_h, stream);
  if (e != cudaSuccess) return e;
  {
    const uint8_t* p[3] = {s->wq, s->wk, s->wv};
    const uint8_t* m[3] = {s->wq_meta, s->wk_meta, s->wv_meta};
    float* y[3] = {q, k, v};
    const uint32_t r[3] = {s->q_rows, s->kv_rows, s->kv_rows};
    e = qg::launch_gemv_multi(s->attn_fmt, 3, p, m, y, r, s->hidden, h, w + L.act_h, stream);
    if (e != cudaSuccess) return e;
  }
  e = qg::launch_act_prepare(q, s->q_rows, w + L.act_q, stream);
  if (e != cudaSuccess) return e;
  e = qg::launch_gemv(s->attn_fmt, s->wo, s->wo_meta, q, w + L.act_q, o, nullptr, nullptr, nullptr,
                      0u, 0u, 0u, s->hidden, s->q_rows, stream);
  if (e != cudaSuccess) return e;
  e = qg::launch_act_prepare(o, s->hidden, w + L.act_o, stream);
  if (e != cudaSuccess) return e;
  {
    const uint8_t* p[2] = {s->wg, s->wu};
    const uint8_t* m[2] = {s->wg_meta, s->wu_meta};
    float* y[2] = {g, u};
    const uint32_t r[2] = {s->ffn, s->ffn};
    e = qg::launch_gemv_multi(s->ffn_fmt, 2, p, m, y, r, s->hidden, o, w + L.act_o, stream);
    if (e != cudaSuccess) return e;
  }
  e = qg::launch_silu_gate_prepare(g, u, s->ffn, a, w + L.act_a, stream);
  if (e != cudaSuccess) return e;
  return qg::launch_gemv(s->down_fmt, s->wd, s->wd_meta, a, w + L.act_a, out, x, nullptr, nullptr,
                         0u, 0u, 0u, s->hidden, s->ffn, stream);
}

cudaError_t qg_layer_slice_batched_workspace_bytes(const qg_layer_slice* s, uint32_t batch,
                                                   size_t* bytes) {
  if (!dims_ok(s) || bytes == nullptr || batch == 0u || batch > 32u) return cudaErrorInvalidValue;
  *bytes = batched_layout(s, batch).total;
  return cudaSuccess;
}

cudaError_t qg_layer_slice_forward_batched(const qg_layer_slice* s, const float* x, float* out,
                                           uint32_t batch, void* workspace, cudaStream_t stream) {
  if (!dims_ok(s) || x == nullptr || out == nullptr || workspace == nullptr || batch == 0u ||
      batch > 32u || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0u) {
    return cudaErrorInvalidValue;
  }
  if (batch == 1u) return qg_layer_slice_forward(s, x, out, workspace, stream);
  const BatchedLayout L = batched_layout(s, batch);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  auto F = [&](size_t off) { return reinterpret_cast<float*>(w + off); };
  void* tc = L.tc != L.total ? w + L.tc : nullptr;
  auto gemm = [&](int fmt, const uint8_t* p, const uint8_t* m, const float* in, float* y, uint32_t rows,
                  uint32_t cols) {
    return qg::launch_batched_gemm(fmt, p, m, in, y, batch, rows, cols, tc, stream);
  };
  cudaError_t e = qg::launch_norm_rows(x, s->norm_weight, s->hidden, s->eps, F(L.h), batch, stream);
  if (e == cudaSuccess) e = gemm(s->attn_fmt, s->wq, s->wq_meta, F(L.h), F(L.q), s->q_rows, s->hidden);
  if (e == cudaSuccess) e = gemm(s->attn_fmt, s->wk, s->wk_meta, F(L.h), F(L.k), s->kv_rows, s->hidden);
  if (e == cudaSuccess) e = gemm(s->attn_fmt, s->wv, s->wv_meta, F(L.h), F(L.v), s->kv_rows, s->hidden);
  if (e == cudaSuccess) e = gemm(s->attn_fmt, s->wo, s->wo_meta, F(L.q), F(L.o), s->hidden, s->q_rows);
  if (e == cudaSuccess) e = gemm(s->ffn_fmt, s->wg, s->wg_meta, F(L.o), F(L.g), s->ffn, s->hidden);
  if (e == cudaSuccess) e = gemm(s->ffn_fmt, s->wu, s->wu_meta, F(L.o), F(L.u), s->ffn, s->hidden);
  if (e == cudaSuccess) e = qg::launch_silu_gate_rows(F(L.g), F(L.u), size_t(batch) * s->ffn, F(L.a), stream);
  if (e == cudaSuccess) e = gemm(s->down_fmt, s->wd, s->wd_meta, F(L.a), F(L.y), s->hidden, s->ffn);
  if (e == cudaSuccess) e = qg::launch_add_rows(x, F(L.y), size_t(batch) * s->hidden, out, stream);
  return e;
}

cudaError_t qg_layer_slice_batched_buffers(const qg_layer_slice* s, uint32_t batch, void* workspace,
                                           qg_layer_slice_views* views) {
  if (!dims_ok(s) || workspace == nullptr || views == nullptr || batch == 0u || batch > 32u) {
    return cudaErrorInvalidValue;
  }
  if (batch == 1u) return qg_layer_slice_buffers(s, workspace, views);
  const BatchedLayout L = batched_layout(s, batch);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  views->h = reinterpret_cast<float*>(w + L.h);
  views->q = reinterpret_cast<float*>(w + L.q);
  views->k = reinterpret_cast<float*>(w + L.k);
  views->v = reinterpret_cast<float*>(w + L.v);
  views->o = reinterpret_cast<float*>(w + L.o);
  views->gate = reinterpret_cast<float*>(w + L.g);
  views->up = reinterpret_cast<float*>(w + L.u);
  views->act = reinterpret_cast<float*>(w + L.a);
  return cudaSuccess;
}

// ---------------------------------------------------------------------------
// Decode-step graphs: capture everything enqueued on `stream` between begin and end
// into one executable graph, uploaded to the device, replayed with one launch.

cudaError_t qg_graph_begin(cudaStream_t stream) {
  return cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal);
}

cudaError_t qg_graph_end(cudaStream_t stream, qg_graph* out) {
  if (out == nullptr) return cudaErrorInvalidValue;
  *out = nullptr;
  auto* g = new (std::nothrow) qg_graph_s();
  if (g == nullptr) return cudaErrorMemoryAllocation;
  cudaError_t e = cudaStreamEndCapture(stream, &g->graph);
  if (e == cudaSuccess) e = cudaGraphInstantiate(&g->exec, g->graph, 0);
  if (e == cudaSuccess) e = cudaGraphUpload(g->exec, stream);
  if (e != cudaSuccess) {
    if (g->exec) cudaGraphExecDestroy(g->exec);
    if (g->graph) cudaGraphDestroy(g->graph);
    delete g;
    return e;
  }
  *out = g;
  return cudaSuccess;
}

cudaError_t qg_graph_launch(qg_graph g, cudaStream_t stream) {
  if (g == nullptr || g->exec == nullptr) return cudaErrorInvalidValue;
  return cudaGraphLaunch(g->exec, stream);
}

cudaError_t qg_graph_destroy(qg_graph g) {
  if (g == nullptr) return cudaSuccess;
  cudaError_t e = cudaSuccess;
  if (g->exec) e = cudaGraphExecDestroy(g->exec);
  if (g->graph) {
    const cudaError_t e2 = cudaGraphDestroy(g->graph);
    if (e == cudaSuccess) e = e2;
  }
  delete g;
  return e;
}

// ---------------------------------------------------------------------------
// One captured graph per batch bucket of the batched slice.  Each bucket owns its padded
// input and output rows and its workspace (allocated at creation, never on a run), and
// the graph of qg_layer_slice_forward_batched at the bucket's batch over them; a run of
// `batch` vectors copies them into the smallest bucket that holds them, replays that
// graph and copies the rows out.  Rows past `batch` hold whatever an earlier run left:
// every row is computed independently, so they cannot change the live rows.

cudaError_t qg_slice_buckets_destroy(qg_slice_buckets b) {
  if (b == nullptr) return cudaSuccess;
  cudaError_t e = cudaSuccess;
  auto keep = [&](cudaError_t r) {
    if (e == cudaSuccess) e = r;
  };
  for (auto& k : b->buckets) {
    if (k.exec) keep(cudaGraphExecDestroy(k.exec));
    if (k.graph) keep(cudaGraphDestroy(k.graph));
    if (k.x) keep(cudaFree(k.x));
    if (k.out) keep(cudaFree(k.out));
    if (k.ws) keep(cudaFree(k.ws));
  }
  delete b;
  return e;
}

cudaError_t qg_slice_buckets_create(const qg_layer_slice* s, const uint32_t* batches, uint32_t n,
                                    cudaStream_t stream, qg_slice_buckets* out) {
  if (out == nullptr || !dims_ok(s) || batches == nullptr || n == 0u || n > 32u) {
    return cudaErrorInvalidValue;
  }
  *out = nullptr;
  for (uint32_t i = 0; i < n; ++i) {
    if (batches[i] == 0u || batches[i] > 32u || (i > 0u && batches[i] <= batches[i - 1u])) {
      return cudaErrorInvalidValue;
    }
  }
  auto* b = new (std::nothrow) qg_slice_buckets_s();
  if (b == nullptr) return cudaErrorMemoryAllocation;
  b->slice = *s;
  // The caller's pending work (e.g. the weights' uploads) first; the warm-up runs and
  // the captures then use a stream of our own (the legacy default stream, which a caller
  // may well pass, cannot be captured).
  cudaError_t e = cudaStreamSynchronize(stream);
  cudaStream_t cap = nullptr;
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete b;
    return e;
  }
  stream = cap;
  for (uint32_t i = 0; i < n && e == cudaSuccess; ++i) {
    b->buckets.emplace_back();
    auto& k = b->buckets.back();
    k.batch = batches[i];
    const size_t rows = size_t(k.batch) * s->hidden * sizeof(float);
    e = cudaMalloc(&k.x, rows);
    if (e == cudaSuccess) e = cudaMalloc(&k.out, rows);
    if (e == cudaSuccess) e = cudaMalloc(&k.ws, batched_layout(s, k.batch).total);
    if (e == cudaSuccess) e = cudaMemsetAsync(k.x, 0, rows, stream);
    // eager run first (kernel attributes, tensor maps), then the capture
    if (e == cudaSuccess) e = qg_layer_slice_forward_batched(&b->slice, k.x, k.out, k.batch, k.ws, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e == cudaSuccess) e = cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
      const cudaError_t fe = qg_layer_slice_forward_batched(&b->slice, k.x, k.out, k.batch, k.ws, stream);
      const cudaError_t ce = cudaStreamEndCapture(stream, &k.graph);
      e = fe != cudaSuccess ? fe : ce;
    }
    if (e == cudaSuccess) e = cudaGraphInstantiate(&k.exec, k.graph, 0);
    if (e == cudaSuccess) e = cudaGraphUpload(k.exec, stream);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  const cudaError_t de = cudaStreamDestroy(cap);
  if (e == cudaSuccess) e = de;
  if (e != cudaSuccess) {
    qg_slice_buckets_destroy(b);
    return e;
  }
  *out = b;
  return cudaSuccess;
}

cudaError_t qg_slice_buckets_bucket(qg_slice_buckets b, uint32_t batch, uint32_t* bucket) {
  if (b == nullptr || bucket == nullptr || batch == 0u) return cudaErrorInvalidValue;
  for (const auto& k : b->buckets) {
    if (k.batch >= batch) {
      *bucket = k.batch;
      return cudaSuccess;
    }
  }
  return cudaErrorInvalidValue;
}

cudaError_t qg_slice_buckets_run(qg_slice_buckets b, const float* x, float* out, uint32_t batch,
                                 cudaStream_t stream) {
  if (b == nullptr || x == nullptr || out == nullptr || batch == 0u) return cudaErrorInvalidValue;
  for (const auto& k : b->buckets) {
    if (k.batch < batch) continue;
    const size_t rows = size_t(batch) * b->slice.hidden * sizeof(float);
    cudaError_t e = cudaMemcpyAsync(k.x, x, rows, cudaMemcpyDeviceToDevice, stream);
    if (e == cudaSuccess) e = cudaGraphLaunch(k.exec, stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, k.out, rows, cudaMemcpyDeviceToDevice, stream);
    return e;
  }
  return cudaErrorInvalidValue;  // larger than the largest bucket
}

}  // extern "C"
