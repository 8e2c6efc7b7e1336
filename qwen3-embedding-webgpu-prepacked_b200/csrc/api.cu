// Host side of the C ABI declared in include/qwa.h.
//
// A context (qwa_ctx) owns, per device: the RoPE cos/sin table
// (src/webgpu/model.ts:76-83, rebuilt when a longer sequence arrives), a
// device status word that kernels write on a failed bounded wait, and a cache
// of launch plans keyed by (cu_seqlens, resolved mode, prefix, window) -- the
// counterpart of the reference engine's plan cache per "batch:sequence"
// (src/webgpu/embedding-engine.ts:70-75). A plan holds the device copy of
// cu_seqlens and the attention work list sorted longest-first.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/qwa.h"
#include "internal.h"
#include "ptx.cuh"

using namespace qwa;

namespace {

constexpr size_t kMaxPlans = 64;

struct Plan {
  int32_t* d_cu = nullptr;
  AttnItem* d_items = nullptr;   // grouped by CTA, then the CTAs' first items (int)
  const int* d_offsets = nullptr;  // inside d_items: CTA c runs items [off[c], off[c+1])
  int n_items = 0;
  int n_ctas = 0;
  int batch = 0;
  int total = 0;
  int max_len = 0;
  ~Plan() {
    if (d_cu) cudaFree(d_cu);
    if (d_items) cudaFree(d_items);
  }
};

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

}  // namespace

struct qwa_ctx {
  int device = 0;
  int sms = 148;  // persistent attention grid size
  std::string error;
  int* d_status = nullptr;
  float* d_rope = nullptr;
  int rope_positions = 0;
  float rope_theta = 0.f;
  std::map<std::vector<int32_t>, std::unique_ptr<Plan>> plans;
  std::vector<std::vector<int32_t>> plan_order;  // insertion order for eviction
  // f16 weights dequantised from Q4_0 tile32 buffers, keyed by (buffer, n, k)
  std::map<std::tuple<const void*, int, int>, __half*> weights;
  std::vector<__half*> retired;  // forgotten copies, freed outside stream capture
  unsigned long long* trace = nullptr;           // QWA_TRACE builds only
  unsigned long long wait_ns = kWaitTimeoutNs;    // bounded-wait limit of the attention kernel
  int skip_load = -1;                             // test hook, see qwa_set_debug
  float* small_ws = nullptr;                      // partial sums of the small-M Q4_0 path
  size_t small_ws_bytes = 0;
};

namespace {

qwa_status fail(qwa_ctx* ctx, qwa_status st, const char* fmt, ...) __attribute__((format(printf, 3, 4)));
qwa_status fail(qwa_ctx* ctx, qwa_status st, const char* fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    ctx->error = buf;
  }
  return st;
}

#define QWA_CUDA(ctx, call)                                                                 \
  do {                                                                                      \
    cudaError_t e_ = (call);                                                                \
    if (e_ != cudaSuccess)                                                                  \
      return fail(ctx, QWA_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_));       \
  } while (0)

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

qwa_status ensure_encode(qwa_ctx* ctx) {
  if (g_encode) return QWA_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
    return fail(ctx, QWA_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return QWA_OK;
}

// 3-D f16 map {128 dims, heads, rows}: head stride 256 B, row stride
// row_stride_bytes; box {64, 1, 128} with 128-byte swizzle, so one load
// lands as 128 rows x 128 B (the canonical SW128 K-major atom layout).
qwa_status make_map(qwa_ctx* ctx, CUtensorMap* map, const void* base, int heads, int64_t rows,
                    int64_t row_stride_bytes, uint32_t box_rows = 128) {
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[2] = {256, static_cast<cuuint64_t>(row_stride_bytes)};
  cuuint32_t box[3] = {64, 1, box_rows};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims,
                        strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(ctx, QWA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return QWA_OK;
}

// 2-D f16 map {inner, rows} with row stride inner*2 bytes, box {64, box_rows},
// 128-byte swizzle (one box = box_rows rows x 128 B, the SW128 K-major atom
// layout the GEMM's descriptors expect). Rows past `rows` read as zero.
qwa_status make_map_2d(qwa_ctx* ctx, CUtensorMap* map, const void* base, int64_t inner,
                       int64_t rows, uint32_t box_rows) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(inner * 2)};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                        strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(ctx, QWA_ERR_CUDA, "cuTensorMapEncodeTiled (2-D) failed (%d)", static_cast<int>(r));
  return QWA_OK;
}

// Output maps of the fused QKV epilogue: boxes of 32 elements x 32 rows
// (64-byte rows, 64-byte swizzle). heads == 0: 2-D {inner, rows}; otherwise
// 3-D {128, heads, rows} with a 256-byte head stride.
qwa_status make_out_map(qwa_ctx* ctx, CUtensorMap* map, void* base, int64_t inner, int heads,
                        int64_t rows, int64_t row_stride_bytes) {
  CUresult r;
  if (heads == 0) {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride_bytes)};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t elem[2] = {1, 1};
    r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims, strides, box, elem,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[2] = {256, static_cast<cuuint64_t>(row_stride_bytes)};
    cuuint32_t box[3] = {32, 1, 32};
    cuuint32_t elem[3] = {1, 1, 1};
    r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, base, dims, strides, box, elem,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS)
    return fail(ctx, QWA_ERR_CUDA, "cuTensorMapEncodeTiled (output) failed (%d)",
                static_cast<int>(r));
  return QWA_OK;
}

qwa_status check_cu(qwa_ctx* ctx, const int32_t* cu, int batch, int* total, int* max_len) {
  if (!cu) return fail(ctx, QWA_ERR_INVALID_ARG, "cu_seqlens_host is NULL");
  if (batch < 1) return fail(ctx, QWA_ERR_INVALID_ARG, "batch must be >= 1 (got %d)", batch);
  if (cu[0] != 0) return fail(ctx, QWA_ERR_INVALID_ARG, "cu_seqlens[0] must be 0");
  int ml = 0;
  for (int b = 0; b < batch; ++b) {
    if (cu[b + 1] < cu[b])
      return fail(ctx, QWA_ERR_INVALID_ARG, "cu_seqlens must be non-decreasing (index %d)", b + 1);
    ml = std::max(ml, cu[b + 1] - cu[b]);
  }
  *total = cu[batch];
  *max_len = ml;
  return QWA_OK;
}

// Work schedule of an attention call. Items are one 128-row query tile x one
// kv head; each gets a cost in key-tile periods (narrow tiles cost less, every
// item pays a fixed fill/drain share). The items are dealt to `sms` CTAs by
// list scheduling (each to the least-loaded CTA) in this order:
// * longest first, which bounds the final imbalance (LPT);
// * for full-causal calls on long requests, request batches first: the items
//   of a few requests whose K/V fit well inside L2 are dealt before the next
//   batch's, so the CTAs running at one time read the same K/V (longest first
//   within a batch). Without it every wave touches every request's K/V and
//   the K/V of earlier keys is re-read from HBM once per query tile.
// Returns the items grouped by CTA and offsets[c]..offsets[c+1] per CTA.
constexpr double kItemOverhead = 0.6;                   // periods per item
constexpr int kGroupMinLen = 2048;                      // full causal, longest request
constexpr int64_t kGroupKvBytes = 48ll << 20;           // K/V bytes per request batch
std::vector<AttnItem> schedule_work(const int32_t* cu, int batch, int sparse, int prefix,
                                    int window, int sms, std::vector<int>* offsets) {
  struct Work {
    double cost;
    int group;
    AttnItem item;
  };
  int max_len = 0;
  for (int b = 0; b < batch; ++b) max_len = std::max(max_len, cu[b + 1] - cu[b]);
  const bool grouped = !sparse && max_len >= kGroupMinLen;
  std::vector<Work> work;
  int group = 0;
  int64_t group_bytes = 0;
  for (int b = 0; b < batch; ++b) {
    const int len = cu[b + 1] - cu[b];
    const int64_t kv_bytes = static_cast<int64_t>(len) * kKVHeads * kHeadDim * 2 * 2;
    if (grouped && group_bytes > 0 && group_bytes + kv_bytes > kGroupKvBytes) {
      ++group;
      group_bytes = 0;
    }
    group_bytes += kv_bytes;
    for (int q0 = 0; q0 < len; q0 += kBlockM) {
      const KeySchedule s = make_key_schedule(q0, len, sparse, prefix, window);
      const int q_last = std::min(q0 + kBlockM, len) - 1;
      double cost = kItemOverhead;
      for (int j = 0; j < s.n; ++j)
        cost += 0.35 + 0.65 * key_tile_width(s, j, q_last, prefix) / double(kBlockN);
      for (int g = 0; g < kKVHeads; ++g)
        work.push_back({cost, grouped ? group : 0, make_int4(cu[b] + q0, q0, len, g)});
    }
  }
  std::stable_sort(work.begin(), work.end(), [](const Work& a, const Work& b) {
    return a.group != b.group ? a.group < b.group : a.cost > b.cost;
  });
  const int n_ctas = static_cast<int>(std::min<size_t>(work.size(), static_cast<size_t>(sms)));
  std::vector<std::vector<int>> per_cta(n_ctas);
  // min-heap of (load, cta)
  std::vector<std::pair<double, int>> heap;
  for (int c = 0; c < n_ctas; ++c) heap.push_back({0.0, c});
  auto cmp = [](const std::pair<double, int>& a, const std::pair<double, int>& b) {
    return a.first != b.first ? a.first > b.first : a.second > b.second;
  };
  std::make_heap(heap.begin(), heap.end(), cmp);
  for (size_t i = 0; i < work.size(); ++i) {
    std::pop_heap(heap.begin(), heap.end(), cmp);
    auto& top = heap.back();
    per_cta[top.second].push_back(static_cast<int>(i));
    top.first += work[i].cost;
    std::push_heap(heap.begin(), heap.end(), cmp);
  }
  std::vector<AttnItem> items;
  items.reserve(work.size());
  offsets->assign(1, 0);
  for (int c = 0; c < n_ctas; ++c) {
    for (int i : per_cta[c]) items.push_back(work[i].item);
    offsets->push_back(static_cast<int>(items.size()));
  }
  return items;
}

// Plan lookup/creation. sparse < 0 requests a plan without attention items
// (the prologue only needs the device cu_seqlens).
qwa_status get_plan(qwa_ctx* ctx, const int32_t* cu, int batch, int sparse, int prefix,
                    int window, cudaStream_t stream, Plan** out) {
  std::vector<int32_t> key;
  key.reserve(batch + 4);
  key.push_back(sparse);
  key.push_back(prefix);
  key.push_back(window);
  key.insert(key.end(), cu, cu + batch + 1);
  auto it = ctx->plans.find(key);
  if (it != ctx->plans.end()) {
    *out = it->second.get();
    return QWA_OK;
  }
  auto plan = std::make_unique<Plan>();
  plan->batch = batch;
  plan->total = cu[batch];
  for (int b = 0; b < batch; ++b) plan->max_len = std::max(plan->max_len, cu[b + 1] - cu[b]);
  QWA_CUDA(ctx, cudaMalloc(&plan->d_cu, sizeof(int32_t) * (batch + 1)));
  QWA_CUDA(ctx, cudaMemcpyAsync(plan->d_cu, cu, sizeof(int32_t) * (batch + 1),
                                cudaMemcpyHostToDevice, stream));
  if (sparse >= 0) {
    std::vector<int> offsets;
    std::vector<AttnItem> items = schedule_work(cu, batch, sparse, prefix, window, ctx->sms,
                                                &offsets);
    plan->n_items = static_cast<int>(items.size());
    plan->n_ctas = static_cast<int>(offsets.size()) - 1;
    if (!items.empty()) {
      const size_t item_bytes = sizeof(AttnItem) * items.size();
      const size_t bytes = item_bytes + sizeof(int) * offsets.size();
      std::vector<uint8_t> host(bytes);
      std::memcpy(host.data(), items.data(), item_bytes);
      std::memcpy(host.data() + item_bytes, offsets.data(), sizeof(int) * offsets.size());
      QWA_CUDA(ctx, cudaMalloc(&plan->d_items, bytes));
      QWA_CUDA(ctx, cudaMemcpyAsync(plan->d_items, host.data(), bytes, cudaMemcpyHostToDevice,
                                    stream));
      // pageable source: the copy is staged before cudaMemcpyAsync returns
      plan->d_offsets = reinterpret_cast<const int*>(
          reinterpret_cast<const uint8_t*>(plan->d_items) + item_bytes);
    }
  }
  if (ctx->plans.size() >= kMaxPlans) {
    // Evict the oldest plan; cudaFree synchronises, so no launch still uses it.
    ctx->plans.erase(ctx->plan_order.front());
    ctx->plan_order.erase(ctx->plan_order.begin());
  }
  *out = plan.get();
  ctx->plan_order.push_back(key);
  ctx->plans.emplace(std::move(key), std::move(plan));
  return QWA_OK;
}

// RoPE table of src/webgpu/model.ts:76-83: angle = pos * theta^(-d/64) in
// double, stored as f32 (cos, sin) pairs.
qwa_status ensure_rope(qwa_ctx* ctx, int positions, float theta, cudaStream_t stream) {
  if (positions <= ctx->rope_positions && theta == ctx->rope_theta) return QWA_OK;
  int n = std::max(positions, 1);
  if (theta == ctx->rope_theta) n = std::max(n, 2 * ctx->rope_positions);
  std::vector<float> host(static_cast<size_t>(n) * 128);
  for (int p = 0; p < n; ++p)
    for (int d = 0; d < 64; ++d) {
      const double angle = static_cast<double>(p) * std::pow(static_cast<double>(theta), -d / 64.0);
      host[(static_cast<size_t>(p) * 64 + d) * 2] = static_cast<float>(std::cos(angle));
      host[(static_cast<size_t>(p) * 64 + d) * 2 + 1] = static_cast<float>(std::sin(angle));
    }
  if (ctx->d_rope) {
    cudaFree(ctx->d_rope);
    ctx->d_rope = nullptr;
    ctx->rope_positions = 0;
  }
  QWA_CUDA(ctx, cudaMalloc(&ctx->d_rope, host.size() * sizeof(float)));
  QWA_CUDA(ctx, cudaMemcpyAsync(ctx->d_rope, host.data(), host.size() * sizeof(float),
                                cudaMemcpyHostToDevice, stream));
  // The pageable copy above has been staged before return; keep ordering simple.
  QWA_CUDA(ctx, cudaStreamSynchronize(stream));
  ctx->rope_positions = n;
  ctx->rope_theta = theta;
  return QWA_OK;
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

qwa_status run_prologue(qwa_ctx* ctx, const void* qkv, int64_t qkv_stride, const float* q_weight,
                        const float* k_weight, void* q_out, void* k_out, const int32_t* d_cu,
                        int batch, int tokens, int padded_sequence, int positions, float eps,
                        float theta, const float* rope_table, cudaStream_t stream) {
  if (!qkv || !q_weight || !k_weight || !q_out || !k_out)
    return fail(ctx, QWA_ERR_INVALID_ARG, "NULL tensor pointer");
  if (qkv_stride < 3072 || qkv_stride % 8 != 0)
    return fail(ctx, QWA_ERR_INVALID_ARG,
                "qkv_stride must be >= 3072 and a multiple of 8 (got %lld)",
                static_cast<long long>(qkv_stride));
  if (!aligned16(qkv) || !aligned16(q_weight) || !aligned16(k_weight) || !aligned16(q_out) ||
      !aligned16(k_out) || (rope_table && !aligned16(rope_table)))
    return fail(ctx, QWA_ERR_INVALID_ARG, "tensor pointers must be 16-byte aligned");
  if (!(eps >= 0.f)) return fail(ctx, QWA_ERR_INVALID_ARG, "eps must be >= 0");
  const float* table = rope_table;
  if (!table) {
    qwa_status st = ensure_rope(ctx, positions, theta, stream);
    if (st != QWA_OK) return st;
    table = ctx->d_rope;
  }
  QWA_CUDA(ctx, launch_qk_norm_rope(static_cast<const __half*>(qkv), qkv_stride, q_weight,
                                    k_weight, reinterpret_cast<const float2*>(table),
                                    static_cast<__half*>(q_out), static_cast<__half*>(k_out), d_cu,
                                    batch, tokens, padded_sequence, eps, stream));
  return QWA_OK;
}

qwa_status run_attention(qwa_ctx* ctx, const void* q, const void* k, const void* v,
                         int64_t v_stride, int64_t v_offset, void* out, const int32_t* cu,
                         int batch, int mode, int prefix, int window, cudaStream_t stream) {
  int total = 0, max_len = 0;
  qwa_status st = check_cu(ctx, cu, batch, &total, &max_len);
  if (st != QWA_OK) return st;
  if (mode < QWA_MODE_AUTO || mode > QWA_MODE_SPARSE)
    return fail(ctx, QWA_ERR_INVALID_ARG, "unknown mode %d", mode);
  if (prefix < 0 || window < 1)
    return fail(ctx, QWA_ERR_INVALID_ARG, "prefix must be >= 0 and window >= 1");
  if (total == 0) return QWA_OK;
  if (!q || !k || !v || !out) return fail(ctx, QWA_ERR_INVALID_ARG, "NULL tensor pointer");
  const void* v_base = static_cast<const __half*>(v) + v_offset;
  if (!aligned16(q) || !aligned16(k) || !aligned16(out) || !aligned16(v_base))
    return fail(ctx, QWA_ERR_INVALID_ARG,
                "q, k, out and v + v_offset must be 16-byte aligned");
  if (v_offset < 0 || v_stride % 8 != 0 || v_stride < v_offset + kKVHeads * kHeadDim)
    return fail(ctx, QWA_ERR_INVALID_ARG,
                "v_stride must be a multiple of 8 and >= v_offset + 1024");
  st = ensure_encode(ctx);
  if (st != QWA_OK) return st;
  const int sparse = resolve_sparse(mode, max_len);
  Plan* plan = nullptr;
  st = get_plan(ctx, cu, batch, sparse, prefix, window, stream, &plan);
  if (st != QWA_OK) return st;
  CUtensorMap tm_q, tm_k, tm_v, tm_o;
  if ((st = make_map(ctx, &tm_q, q, kQHeads, total, kQHeads * kHeadDim * 2)) != QWA_OK) return st;
  if ((st = make_map(ctx, &tm_o, out, kQHeads, total, kQHeads * kHeadDim * 2, kOutBoxRows)) != QWA_OK) return st;
  if ((st = make_map(ctx, &tm_k, k, kKVHeads, total, kKVHeads * kHeadDim * 2)) != QWA_OK) return st;
  if ((st = make_map(ctx, &tm_v, v_base, kKVHeads, total, v_stride * 2)) != QWA_OK) return st;
  AttnArgs args;
  args.items = plan->d_items;
  args.out = static_cast<__half*>(out);
  args.sparse = sparse;
  args.prefix = prefix;
  args.window = window;
  args.scale_log2 = kScale * kLog2e;
  args.status = ctx->d_status;
  args.trace = ctx->trace;
  args.wait_ns = ctx->wait_ns;
  args.skip_load = ctx->skip_load;
  args.cta_offsets = plan->d_offsets;
  args.num_ctas = plan->n_ctas;
  QWA_CUDA(ctx, launch_attention(tm_q, tm_k, tm_v, tm_o, args, plan->n_items, stream));
  return QWA_OK;
}

}  // namespace

extern "C" {

const char* qwa_version(void) { return "qwa 0.1.0 (sm_100a tcgen05)"; }

const char* qwa_status_string(qwa_status s) {
  switch (s) {
    case QWA_OK: return "ok";
    case QWA_ERR_INVALID_ARG: return "invalid argument";
    case QWA_ERR_UNSUPPORTED: return "unsupported";
    case QWA_ERR_CUDA: return "CUDA error";
    case QWA_ERR_TIMEOUT: return "device wait timed out";
    case QWA_ERR_NO_DEVICE: return "no CUDA device";
  }
  return "unknown status";
}

const char* qwa_last_error(const qwa_ctx* ctx) { return ctx ? ctx->error.c_str() : ""; }

qwa_status qwa_create(int device, qwa_ctx** out) {
  if (!out) return QWA_ERR_INVALID_ARG;
  *out = nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    return QWA_ERR_NO_DEVICE;
  }
  if (device < 0 || device >= count) return QWA_ERR_INVALID_ARG;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return QWA_ERR_CUDA;
  if (prop.major != 10) return QWA_ERR_UNSUPPORTED;  // built for sm_100a only
  DeviceGuard guard(device);
  auto ctx = std::make_unique<qwa_ctx>();
  ctx->device = device;
  ctx->sms = prop.multiProcessorCount;
  if (cudaMalloc(&ctx->d_status, sizeof(int)) != cudaSuccess) return QWA_ERR_CUDA;
  if (cudaMemset(ctx->d_status, 0, sizeof(int)) != cudaSuccess) return QWA_ERR_CUDA;
  if (ensure_encode(ctx.get()) != QWA_OK) return QWA_ERR_CUDA;
  *out = ctx.release();
  return QWA_OK;
}

qwa_status qwa_destroy(qwa_ctx* ctx) {
  if (!ctx) return QWA_OK;
  {
    DeviceGuard guard(ctx->device);
    cudaDeviceSynchronize();
    ctx->plans.clear();
    for (auto& w : ctx->weights) cudaFree(w.second);
    ctx->weights.clear();
    for (__half* w : ctx->retired) cudaFree(w);
    ctx->retired.clear();
    if (ctx->d_rope) cudaFree(ctx->d_rope);
    if (ctx->d_status) cudaFree(ctx->d_status);
    if (ctx->small_ws) cudaFree(ctx->small_ws);
  }
  delete ctx;
  return QWA_OK;
}

qwa_status qwa_set_debug(qwa_ctx* ctx, int64_t wait_limit_ns, int skip_kv_load) {
  if (!ctx || skip_kv_load < -1) return QWA_ERR_INVALID_ARG;
  ctx->wait_ns = wait_limit_ns > 0 ? static_cast<unsigned long long>(wait_limit_ns)
                                   : kWaitTimeoutNs;
  ctx->skip_load = skip_kv_load;
  return QWA_OK;
}

// status word of qwa_attention_noalloc on the current device (noalloc.cu)
qwa_status qwa_noalloc_status(void* stream);

qwa_status qwa_check(qwa_ctx* ctx, void* stream) {
  if (!ctx) return qwa_noalloc_status(stream);
  DeviceGuard guard(ctx->device);
  QWA_CUDA(ctx, cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  int code = 0;
  QWA_CUDA(ctx, cudaMemcpy(&code, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost));
  if (code != 0) {
    QWA_CUDA(ctx, cudaMemset(ctx->d_status, 0, sizeof(int)));
    return fail(ctx, QWA_ERR_TIMEOUT, "device-side bounded wait timed out (code 0x%x)", code);
  }
  return QWA_OK;
}

qwa_status qwa_qk_norm_rope(qwa_ctx* ctx, const void* qkv, int64_t qkv_stride,
                            const float* q_weight, const float* k_weight, void* q_out,
                            void* k_out, const int32_t* cu_seqlens_host, int batch, float eps,
                            float theta, const float* rope_table, void* stream) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  DeviceGuard guard(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int total = 0, max_len = 0;
  qwa_status st = check_cu(ctx, cu_seqlens_host, batch, &total, &max_len);
  if (st != QWA_OK) return st;
  if (total == 0) return QWA_OK;
  Plan* plan = nullptr;
  st = get_plan(ctx, cu_seqlens_host, batch, -1, 0, 0, s, &plan);
  if (st != QWA_OK) return st;
  return run_prologue(ctx, qkv, qkv_stride, q_weight, k_weight, q_out, k_out, plan->d_cu, batch,
                      total, 0, max_len, eps, theta, rope_table, s);
}

qwa_status qwa_qk_norm_rope_padded(qwa_ctx* ctx, const void* qkv, int64_t qkv_stride,
                                   const float* q_weight, const float* k_weight, void* q_out,
                                   void* k_out, int tokens, int sequence, float eps, float theta,
                                   const float* rope_table, void* stream) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  DeviceGuard guard(ctx->device);
  if (tokens < 0 || sequence < 1)
    return fail(ctx, QWA_ERR_INVALID_ARG, "tokens must be >= 0 and sequence >= 1");
  if (tokens == 0) return QWA_OK;
  return run_prologue(ctx, qkv, qkv_stride, q_weight, k_weight, q_out, k_out, nullptr, 1, tokens,
                      sequence, std::min(sequence, tokens), eps, theta, rope_table,
                      static_cast<cudaStream_t>(stream));
}

namespace {

// CTA-pair GEMM for large M (QWA_GEMM_PAIR=0 / 1 forces one shape).
bool gemm_pair(int m) {
  static const int forced = [] {
    const char* e = std::getenv("QWA_GEMM_PAIR");
    return e ? std::atoi(e) : -1;
  }();
  if (forced >= 0) return forced != 0;
  return m >= kGemmPairMinRows;
}

qwa_status check_matmul_shape(qwa_ctx* ctx, int m, int n, int k) {
  if (m < 0) return fail(ctx, QWA_ERR_INVALID_ARG, "m must be >= 0");
  if (n < 256 || n % 256 != 0)
    return fail(ctx, QWA_ERR_UNSUPPORTED, "n must be a positive multiple of 256 (got %d)", n);
  if (k < 64 || k % 64 != 0)
    return fail(ctx, QWA_ERR_UNSUPPORTED, "k must be a positive multiple of 64 (got %d)", k);
  return QWA_OK;
}

// glu: the gate_up form with the SwiGLU in the epilogue (output [m, n / 2]).
qwa_status run_matmul(qwa_ctx* ctx, const void* input, const void* weight, void* output, int m,
                      int n, int k, cudaStream_t stream, bool glu = false) {
  if (!input || !weight || !output) return fail(ctx, QWA_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(input) || !aligned16(weight) || !aligned16(output))
    return fail(ctx, QWA_ERR_INVALID_ARG, "tensor pointers must be 16-byte aligned");
  qwa_status st = ensure_encode(ctx);
  if (st != QWA_OK) return st;
  const bool pair = gemm_pair(m);
  CUtensorMap tm_a, tm_w, tm_out;
  if ((st = make_map_2d(ctx, &tm_a, input, k, m, 128)) != QWA_OK) return st;
  if ((st = make_map_2d(ctx, &tm_w, weight, k, n, kGemmWBoxRows(pair))) != QWA_OK) return st;
  if ((st = make_map_2d(ctx, &tm_out, output, glu ? n / 2 : n, m, 32)) != QWA_OK) return st;
  if (glu)
    QWA_CUDA(ctx, launch_gemm_glu(tm_a, tm_w, tm_out, static_cast<__half*>(output), m, n, k,
                                  ctx->d_status, pair, stream));
  else
    QWA_CUDA(ctx, launch_gemm_f16(tm_a, tm_w, tm_out, static_cast<__half*>(output), m, n, k,
                                  ctx->d_status, pair, stream));
  return QWA_OK;
}

// Small batches (m <= 64 rows): the Q4_0 records are read directly (no f16
// copy), K split across CTAs, partial sums in a context workspace.
qwa_status run_q40_small(qwa_ctx* ctx, const void* input, const void* packed, void* output, int m,
                         int n, int k, cudaStream_t stream) {
  if (!input || !output) return fail(ctx, QWA_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(input) || !aligned16(output))
    return fail(ctx, QWA_ERR_INVALID_ARG, "tensor pointers must be 16-byte aligned");
  qwa_status st = ensure_encode(ctx);
  if (st != QWA_OK) return st;
  const int splits = q40_small_splits(n, k, ctx->sms);
  const size_t need = sizeof(float) * static_cast<size_t>(splits) * m * n;
  if (need > ctx->small_ws_bytes) {
    // grows once per larger shape; synchronises (cudaFree) outside any capture
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
      return fail(ctx, QWA_ERR_UNSUPPORTED,
                  "the small-batch Q4_0 workspace must grow: make one call of this shape "
                  "before capturing");
    if (ctx->small_ws) cudaFree(ctx->small_ws);
    ctx->small_ws = nullptr;
    ctx->small_ws_bytes = 0;
    QWA_CUDA(ctx, cudaMalloc(&ctx->small_ws, need));
    ctx->small_ws_bytes = need;
  }
  CUtensorMap tm_x;
  const uint32_t mpad = static_cast<uint32_t>((m + 15) / 16 * 16);
  if ((st = make_map_2d(ctx, &tm_x, input, k, m, mpad)) != QWA_OK) return st;
  QWA_CUDA(ctx, launch_q40_small_gemm(tm_x, static_cast<const uint8_t*>(packed),
                                      static_cast<__half*>(output), m, n, k, splits,
                                      ctx->small_ws, ctx->d_status, stream));
  return QWA_OK;
}

qwa_status check_q40(qwa_ctx* ctx, const void* packed, int n, int k) {
  if (!packed) return fail(ctx, QWA_ERR_INVALID_ARG, "NULL weight pointer");
  if (n < 1 || k < 32 || k % 32 != 0)
    return fail(ctx, QWA_ERR_INVALID_ARG, "n must be >= 1 and k a positive multiple of 32");
  if (reinterpret_cast<uintptr_t>(packed) & 3u)
    return fail(ctx, QWA_ERR_INVALID_ARG, "packed weights must be 4-byte aligned");
  return QWA_OK;
}

}  // namespace

qwa_status qwa_q40_dequantize(qwa_ctx* ctx, const void* packed, int n, int k, void* weight,
                              void* stream) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  DeviceGuard guard(ctx->device);
  qwa_status st = check_q40(ctx, packed, n, k);
  if (st != QWA_OK) return st;
  if (!weight || !aligned16(weight))
    return fail(ctx, QWA_ERR_INVALID_ARG, "weight must be a 16-byte aligned pointer");
  QWA_CUDA(ctx, launch_q40_tile32_dequant(static_cast<const uint8_t*>(packed), n, k,
                                          static_cast<__half*>(weight),
                                          static_cast<cudaStream_t>(stream)));
  return QWA_OK;
}

qwa_status qwa_matmul_swiglu(qwa_ctx* ctx, const void* input, const void* weight, void* output,
                             int m, int n, int k, void* stream) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  DeviceGuard guard(ctx->device);
  qwa_status st = check_matmul_shape(ctx, m, n, k);
  if (st != QWA_OK) return st;
  if (m == 0) return QWA_OK;
  return run_matmul(ctx, input, weight, output, m, n, k, static_cast<cudaStream_t>(stream), true);
}

qwa_status qwa_matmul(qwa_ctx* ctx, const void* input, const void* weight, void* output, int m,
                      int n, int k, void* stream) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  DeviceGuard guard(ctx->device);
  qwa_status st = check_matmul_shape(ctx, m, n, k);
  if (st != QWA_OK) return st;
  if (m == 0) return QWA_OK;
  return run_matmul(ctx, input, weight, output, m, n, k, static_cast<cudaStream_t>(stream));
}

namespace {

// f16 copy of a Q4_0 tile32 matrix owned by the context (made on first use).
qwa_status cached_q40(qwa_ctx* ctx, const void* packed, int n, int k, cudaStream_t s,
                      __half** out) {
  if (!ctx->retired.empty()) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusNone) {
      // cudaFree waits for the device, so no launch still reads these
      for (__half* w : ctx->retired) cudaFree(w);
      ctx->retired.clear();
    }
  }
  const auto key = std::make_tuple(packed, n, k);
  auto it = ctx->weights.find(key);
  if (it != ctx->weights.end()) {
    *out = it->second;
    return QWA_OK;
  }
  __half* w = nullptr;
  QWA_CUDA(ctx, cudaMalloc(&w, static_cast<size_t>(n) * k * sizeof(__half)));
  ctx->weights[key] = w;
  QWA_CUDA(ctx, launch_q40_tile32_dequant(static_cast<const uint8_t*>(packed), n, k, w, s));
  *out = w;
  return QWA_OK;
}

qwa_status run_qkv_projection(qwa_ctx* ctx, const void* input, const void* weight, int k,
                              const float* q_weight, const float* k_weight, void* q_out,
                              void* k_out, void* v_out, const int32_t* cu, int batch, float eps,
                              float theta, const float* rope_table, cudaStream_t s) {
  int total = 0, max_len = 0;
  qwa_status st = check_cu(ctx, cu, batch, &total, &max_len);
  if (st != QWA_OK) return st;
  if (k < 64 || k % 64 != 0)
    return fail(ctx, QWA_ERR_UNSUPPORTED, "k must be a positive multiple of 64 (got %d)", k);
  if (!(eps >= 0.f)) return fail(ctx, QWA_ERR_INVALID_ARG, "eps must be >= 0");
  if (total == 0) return QWA_OK;
  if (!input || !weight || !q_weight || !k_weight || !q_out || !k_out || !v_out)
    return fail(ctx, QWA_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(input) || !aligned16(weight) || !aligned16(q_weight) || !aligned16(k_weight) ||
      !aligned16(q_out) || !aligned16(k_out) || !aligned16(v_out) ||
      (rope_table && !aligned16(rope_table)))
    return fail(ctx, QWA_ERR_INVALID_ARG, "tensor pointers must be 16-byte aligned");
  if ((st = ensure_encode(ctx)) != QWA_OK) return st;
  Plan* plan = nullptr;
  if ((st = get_plan(ctx, cu, batch, -1, 0, 0, s, &plan)) != QWA_OK) return st;
  const float* table = rope_table;
  if (!table) {
    if ((st = ensure_rope(ctx, max_len, theta, s)) != QWA_OK) return st;
    table = ctx->d_rope;
  }
  CUtensorMap tm_a, tm_w;
  if ((st = make_map_2d(ctx, &tm_a, input, k, total, 128)) != QWA_OK) return st;
  const bool pair = gemm_pair(total);
  if ((st = make_map_2d(ctx, &tm_w, weight, k, 4096, kGemmWBoxRows(pair))) != QWA_OK) return st;
  QkvEpilogue e;
  e.q_out = static_cast<__half*>(q_out);
  e.k_out = static_cast<__half*>(k_out);
  e.v_out = static_cast<__half*>(v_out);
  e.q_weight = q_weight;
  e.k_weight = k_weight;
  e.table = reinterpret_cast<const float2*>(table);
  e.cu = plan->d_cu;
  e.batch = batch;
  e.eps = eps;
  CUtensorMap tm_vo = tm_a, tm_qo = tm_a, tm_ko = tm_a;  // single-CTA launches store directly
  if (pair) {
    if ((st = make_out_map(ctx, &tm_vo, v_out, 1024, 0, total, 1024 * 2)) != QWA_OK) return st;
    if ((st = make_out_map(ctx, &tm_qo, q_out, 128, 16, total, 16 * 128 * 2)) != QWA_OK) return st;
    if ((st = make_out_map(ctx, &tm_ko, k_out, 128, 8, total, 8 * 128 * 2)) != QWA_OK) return st;
  }
  QWA_CUDA(ctx, launch_gemm_qkv(tm_a, tm_w, tm_vo, tm_qo, tm_ko, total, k, e, ctx->d_status, pair,
                                s));
  return QWA_OK;
}

}  // namespace

qwa_status qwa_qkv_projection(qwa_ctx* ctx, const void* input, const void* weight, int k,
                              const float* q_weight, const float* k_weight, void* q_out,
                              void* k_out, void* v_out, const int32_t* cu_seqlens_host,
                              int batch, float eps, float theta, const float* rope_table,
                              void* stream) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  DeviceGuard guard(ctx->device);
  return run_qkv_projection(ctx, input, weight, k, q_weight, k_weight, q_out, k_out, v_out,
                            cu_seqlens_host, batch, eps, theta, rope_table,
                            static_cast<cudaStream_t>(stream));
}

qwa_status qwa_q40_qkv_projection(qwa_ctx* ctx, const void* input, const void* packed, int k,
                                  const float* q_weight, const float* k_weight, void* q_out,
                                  void* k_out, void* v_out, const int32_t* cu_seqlens_host,
                                  int batch, float eps, float theta, const float* rope_table,
                                  void* stream) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  DeviceGuard guard(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  qwa_status st = check_q40(ctx, packed, 4096, k);
  if (st != QWA_OK) return st;
  __half* w = nullptr;
  if ((st = cached_q40(ctx, packed, 4096, k, s, &w)) != QWA_OK) return st;
  return run_qkv_projection(ctx, input, w, k, q_weight, k_weight, q_out, k_out, v_out,
                            cu_seqlens_host, batch, eps, theta, rope_table, s);
}

qwa_status qwa_q40_matmul(qwa_ctx* ctx, const void* input, const void* packed, void* output,
                          int m, int n, int k, void* stream) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  DeviceGuard guard(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  qwa_status st = check_matmul_shape(ctx, m, n, k);
  if (st == QWA_OK) st = check_q40(ctx, packed, n, k);
  if (st != QWA_OK) return st;
  if (m == 0) return QWA_OK;
  // Few rows on a matrix of few output rows: the records are read directly
  // (measured 1.5-1.9x faster than the f16 GEMM at n = 1024, k = 2048 / 3072;
  // on par or slower for n = 4096 / 6144, where the f16 GEMM keeps enough CTAs
  // busy without splitting K).
  if (m <= kQ40SmallMaxRows && n <= 2048)
    return run_q40_small(ctx, input, packed, output, m, n, k, s);
  __half* w = nullptr;
  if ((st = cached_q40(ctx, packed, n, k, s, &w)) != QWA_OK) return st;
  return run_matmul(ctx, input, w, output, m, n, k, s);
}

qwa_status qwa_q40_forget(qwa_ctx* ctx, const void* packed) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  // No synchronisation or free here (this may run while a stream is being
  // captured): the copies move to a list freed by the next Q4_0 call made
  // outside a capture, or by qwa_destroy.
  for (auto it = ctx->weights.begin(); it != ctx->weights.end();) {
    if (std::get<0>(it->first) == packed) {
      ctx->retired.push_back(it->second);
      it = ctx->weights.erase(it);
    } else {
      ++it;
    }
  }
  return QWA_OK;
}

qwa_status qwa_rms_norm(qwa_ctx* ctx, void* x, const void* residual, const float* weight,
                        void* normalized, int rows, int width, float eps, int has_residual,
                        void* stream) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  DeviceGuard guard(ctx->device);
  if (rows < 0) return fail(ctx, QWA_ERR_INVALID_ARG, "rows must be >= 0");
  if (width < 8 || width % 8 != 0)
    return fail(ctx, QWA_ERR_INVALID_ARG, "width must be a positive multiple of 8 (got %d)", width);
  if (!(eps >= 0.f)) return fail(ctx, QWA_ERR_INVALID_ARG, "eps must be >= 0");
  if (rows == 0) return QWA_OK;
  if (!x || !weight || !normalized || (has_residual && !residual))
    return fail(ctx, QWA_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(x) || !aligned16(weight) || !aligned16(normalized) ||
      (has_residual && !aligned16(residual)))
    return fail(ctx, QWA_ERR_INVALID_ARG, "tensor pointers must be 16-byte aligned");
  QWA_CUDA(ctx, launch_rms_norm(static_cast<__half*>(x), static_cast<const __half*>(residual),
                                weight, static_cast<__half*>(normalized), rows, width,
                                has_residual != 0, eps, static_cast<cudaStream_t>(stream)));
  return QWA_OK;
}

qwa_status qwa_swiglu(qwa_ctx* ctx, const void* combined, void* out, int rows, int width,
                      void* stream) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  DeviceGuard guard(ctx->device);
  if (rows < 0) return fail(ctx, QWA_ERR_INVALID_ARG, "rows must be >= 0");
  if (width < 8 || width % 8 != 0)
    return fail(ctx, QWA_ERR_INVALID_ARG, "width must be a positive multiple of 8 (got %d)", width);
  if (rows == 0) return QWA_OK;
  if (!combined || !out) return fail(ctx, QWA_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(combined) || !aligned16(out))
    return fail(ctx, QWA_ERR_INVALID_ARG, "tensor pointers must be 16-byte aligned");
  QWA_CUDA(ctx, launch_swiglu(static_cast<const __half*>(combined), static_cast<__half*>(out),
                              rows, width, static_cast<cudaStream_t>(stream)));
  return QWA_OK;
}

qwa_status qwa_embedding_lookup_q6k(qwa_ctx* ctx, const uint32_t* ids_device, const void* table,
                                    int vocab, void* out, int tokens, int width, void* stream) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  DeviceGuard guard(ctx->device);
  if (tokens < 0 || vocab < 0) return fail(ctx, QWA_ERR_INVALID_ARG, "tokens and vocab must be >= 0");
  if (width < 256 || width % 256 != 0)
    return fail(ctx, QWA_ERR_INVALID_ARG, "width must be a positive multiple of 256 (got %d)",
                width);
  if (tokens == 0) return QWA_OK;
  if (!ids_device || !out || (vocab > 0 && !table))
    return fail(ctx, QWA_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(out) || (reinterpret_cast<uintptr_t>(table) & 1u) ||
      (reinterpret_cast<uintptr_t>(ids_device) & 3u))
    return fail(ctx, QWA_ERR_INVALID_ARG,
                "out must be 16-byte, table 2-byte and ids 4-byte aligned");
  QWA_CUDA(ctx, launch_q6k_embedding(ids_device, static_cast<const uint8_t*>(table), vocab,
                                     static_cast<__half*>(out), tokens, width,
                                     static_cast<cudaStream_t>(stream)));
  return QWA_OK;
}

qwa_status qwa_last_token_pool(qwa_ctx* ctx, const void* hidden, int width, float* out,
                               const int32_t* cu_seqlens_host, int batch, void* stream) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  DeviceGuard guard(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int total = 0, max_len = 0;
  qwa_status st = check_cu(ctx, cu_seqlens_host, batch, &total, &max_len);
  if (st != QWA_OK) return st;
  if (width < 8 || width % 8 != 0)
    return fail(ctx, QWA_ERR_INVALID_ARG, "width must be a positive multiple of 8 (got %d)", width);
  if (!out || (total > 0 && !hidden)) return fail(ctx, QWA_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(out) || (hidden && !aligned16(hidden)))
    return fail(ctx, QWA_ERR_INVALID_ARG, "hidden and out must be 16-byte aligned");
  Plan* plan = nullptr;
  st = get_plan(ctx, cu_seqlens_host, batch, -1, 0, 0, s, &plan);
  if (st != QWA_OK) return st;
  QWA_CUDA(ctx, launch_last_token_pool(static_cast<const __half*>(hidden), width, plan->d_cu,
                                       nullptr, 0, batch, out, s));
  return QWA_OK;
}

qwa_status qwa_last_token_pool_padded(qwa_ctx* ctx, const void* hidden,
                                      const uint32_t* lengths_device, float* out, int batch,
                                      int sequence, int width, void* stream) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  DeviceGuard guard(ctx->device);
  if (batch < 1 || sequence < 1)
    return fail(ctx, QWA_ERR_INVALID_ARG, "batch and sequence must be >= 1");
  if (width < 8 || width % 8 != 0)
    return fail(ctx, QWA_ERR_INVALID_ARG, "width must be a positive multiple of 8 (got %d)", width);
  if (!hidden || !lengths_device || !out)
    return fail(ctx, QWA_ERR_INVALID_ARG, "NULL tensor pointer");
  if (!aligned16(out) || !aligned16(hidden))
    return fail(ctx, QWA_ERR_INVALID_ARG, "hidden and out must be 16-byte aligned");
  QWA_CUDA(ctx, launch_last_token_pool(static_cast<const __half*>(hidden), width, nullptr,
                                       lengths_device, sequence, batch, out,
                                       static_cast<cudaStream_t>(stream)));
  return QWA_OK;
}

qwa_status qwa_attention(qwa_ctx* ctx, const void* q, const void* k, const void* v,
                         int64_t v_stride, int64_t v_offset, void* out,
                         const int32_t* cu_seqlens_host, int batch, int mode, int prefix,
                         int window, void* stream) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  DeviceGuard guard(ctx->device);
  return run_attention(ctx, q, k, v, v_stride, v_offset, out, cu_seqlens_host, batch, mode, prefix,
                       window, static_cast<cudaStream_t>(stream));
}

qwa_status qwa_attention_padded(qwa_ctx* ctx, const void* q, const void* k, const void* v,
                                void* out, int batch, int sequence, int q_heads, int kv_heads,
                                int64_t value_stride, int64_t value_offset, void* stream) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  if (q_heads != kQHeads || kv_heads != kKVHeads)
    return fail(ctx, QWA_ERR_UNSUPPORTED, "only 16 query heads / 8 kv heads are supported");
  if (batch < 1 || sequence < 1)
    return fail(ctx, QWA_ERR_INVALID_ARG, "batch and sequence must be >= 1");
  if (static_cast<int64_t>(batch) * sequence > 0x7fffffff)
    return fail(ctx, QWA_ERR_INVALID_ARG, "batch * sequence overflows int32");
  std::vector<int32_t> cu(batch + 1);
  for (int b = 0; b <= batch; ++b) cu[b] = b * sequence;
  DeviceGuard guard(ctx->device);
  return run_attention(ctx, q, k, v, value_stride, value_offset, out, cu.data(), batch,
                       QWA_MODE_AUTO, 176, 432, static_cast<cudaStream_t>(stream));
}

qwa_status qwa_prefill_attention_layer(qwa_ctx* ctx, const void* qkv, int64_t qkv_stride,
                                       const float* q_weight, const float* k_weight, void* q_buf,
                                       void* k_buf, void* out, const int32_t* cu_seqlens_host,
                                       int batch, int mode, int prefix, int window, float eps,
                                       float theta, void* stream) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  if (qkv_stride < 4096)
    return fail(ctx, QWA_ERR_INVALID_ARG, "qkv_stride must be >= 4096 (q, k and v columns)");
  qwa_status st = qwa_qk_norm_rope(ctx, qkv, qkv_stride, q_weight, k_weight, q_buf, k_buf,
                                   cu_seqlens_host, batch, eps, theta, nullptr, stream);
  if (st != QWA_OK) return st;
  DeviceGuard guard(ctx->device);
  return run_attention(ctx, q_buf, k_buf, qkv, qkv_stride, 3072, out, cu_seqlens_host, batch, mode,
                       prefix, window, static_cast<cudaStream_t>(stream));
}

qwa_status qwa_attention_work(const int32_t* cu, int batch, int mode, int prefix, int window,
                              int64_t* kept_pairs, int64_t* visited_tiles) {
  int total = 0, max_len = 0;
  qwa_status st = check_cu(nullptr, cu, batch, &total, &max_len);
  if (st != QWA_OK) return st;
  if (prefix < 0 || window < 1) return QWA_ERR_INVALID_ARG;
  const int sparse = resolve_sparse(mode, max_len);
  int64_t pairs = 0, tiles = 0;
  for (int b = 0; b < batch; ++b) {
    const int len = cu[b + 1] - cu[b];
    for (int qi = 0; qi < len; ++qi) {
      if (!sparse) {
        pairs += qi + 1;
      } else {
        // keys [0, min(prefix, q+1)) plus (q - window, q] minus their overlap
        const int64_t lo = std::max(0, qi - window + 1);
        const int64_t pre = std::min(prefix, qi + 1);
        const int64_t win = qi + 1 - lo;
        const int64_t overlap = std::max<int64_t>(0, pre - lo);
        pairs += pre + win - overlap;
      }
    }
    for (int q0 = 0; q0 < len; q0 += kBlockM)
      tiles += make_key_schedule(q0, len, sparse, prefix, window).n;
  }
  if (kept_pairs) *kept_pairs = pairs;
  if (visited_tiles) *visited_tiles = tiles * kKVHeads;  // per kv group (two q heads each)
  return QWA_OK;
}

qwa_status qwa_selftest_tile(qwa_ctx* ctx, const void* a, const void* b, const void* vt, float* c,
                             float* d, void* stream) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  if (!a || !b || !vt || !c || !d) return fail(ctx, QWA_ERR_INVALID_ARG, "NULL pointer");
  if (!aligned16(a) || !aligned16(b) || !aligned16(vt))
    return fail(ctx, QWA_ERR_INVALID_ARG, "inputs must be 16-byte aligned");
  DeviceGuard guard(ctx->device);
  qwa_status st = ensure_encode(ctx);
  if (st != QWA_OK) return st;
  CUtensorMap ta, tb, tv;
  if ((st = make_map(ctx, &ta, a, 1, 128, 256)) != QWA_OK) return st;
  if ((st = make_map(ctx, &tb, b, 1, 128, 256)) != QWA_OK) return st;
  if ((st = make_map(ctx, &tv, vt, 1, 128, 256)) != QWA_OK) return st;
  QWA_CUDA(ctx, launch_selftest_tile(ta, tb, tv, c, d, ctx->d_status,
                                     static_cast<cudaStream_t>(stream)));
  return QWA_OK;
}

#ifdef QWA_TRACE
// Trace builds only (not part of include/qwa.h): attention launches record a
// clock64 timeline of the first CTAs into `trace` (device buffer of
// kTraceCtas * kTraceEvents * kTraceIters u64), or stop recording with NULL.
QWA_API qwa_status qwa_debug_set_trace(qwa_ctx* ctx, unsigned long long* trace) {
  if (!ctx) return QWA_ERR_INVALID_ARG;
  ctx->trace = trace;
  return QWA_OK;
}
#endif

}  // extern "C"
