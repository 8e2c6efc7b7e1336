// qwa_attention_noalloc: the attention kernel with its scratch memory in a
// fixed, library-owned device array instead of context allocations.
//
// Who needs it: callers that must not allocate device memory at run time,
// for example a host runtime that hands the library a pre-planned arena and
// forbids cudaMalloc/cudaFree on its serving path (they synchronise the device
// and can fail under memory pressure), or an embedding process that has not
// created a qwa_ctx. This entry point takes no context and calls no
// cudaMalloc, cudaFree or allocating library routine.
//
// Scratch: the attention work list (one 16-byte item per 128-row query tile
// per kv head) and the kernels' status word live in g_scratch below, a
// file-scope device array of kScratchBytes. Every GPU that loads the library
// holds it until the process exits. A call whose work list does not fit is
// rejected with QWA_ERR_INVALID_ARG before anything is launched.
//
// The array's name is only a host-side stand-in; the device address is
// obtained once per device with cudaGetSymbolAddress, on the first call made
// with that device current. Make that first call before any stream capture.
// All calls share the one array and it keeps the last call's contents: the
// status word is cleared on every call, and calls whose launches overlap on
// the GPU (different streams, no ordering between them) race on the work
// list and produce wrong results.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "../../include/qwa.h"
#include "internal.h"

using namespace qwa;

namespace {

constexpr size_t kScratchBytes = 1u << 20;  // 1 MiB
constexpr size_t kStatusBytes = 256;        // status word, padded
constexpr size_t kMaxItems = (kScratchBytes - kStatusBytes) / sizeof(AttnItem);

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices] = {};
PFN_cuTensorMapEncodeTiled_v12000 g_encode_na = nullptr;

qwa_status setup_device(int device, unsigned char** out) {
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_encode_na) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return QWA_ERR_CUDA;
    g_encode_na = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  if (!g_scratch_ptr[device]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || !p) return QWA_ERR_CUDA;
    g_scratch_ptr[device] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch_ptr[device]);
  return QWA_OK;
}

bool map3d(CUtensorMap* map, const void* base, int heads, int64_t rows, int64_t row_stride) {
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[2] = {256, static_cast<cuuint64_t>(row_stride)};
  cuuint32_t box[3] = {64, 1, 128};
  cuuint32_t elem[3] = {1, 1, 1};
  return g_encode_na(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims,
                     strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" qwa_status qwa_attention_noalloc(const void* q, const void* k, const void* v,
                                            int64_t v_stride, int64_t v_offset, void* out,
                                            const int32_t* cu, int batch, int mode, int prefix,
                                            int window, void* stream) {
  if (!cu || batch < 1 || cu[0] != 0) return QWA_ERR_INVALID_ARG;
  int max_len = 0;
  for (int b = 0; b < batch; ++b) {
    if (cu[b + 1] < cu[b]) return QWA_ERR_INVALID_ARG;
    max_len = cu[b + 1] - cu[b] > max_len ? cu[b + 1] - cu[b] : max_len;
  }
  const int total = cu[batch];
  if (mode < QWA_MODE_AUTO || mode > QWA_MODE_SPARSE || prefix < 0 || window < 1)
    return QWA_ERR_INVALID_ARG;
  if (total == 0) return QWA_OK;
  if (!q || !k || !v || !out) return QWA_ERR_INVALID_ARG;
  const void* v_base = static_cast<const __half*>(v) + v_offset;
  if (!aligned16(q) || !aligned16(k) || !aligned16(out) || !aligned16(v_base) || v_offset < 0 ||
      v_stride % 8 != 0 || v_stride < v_offset + kKVHeads * kHeadDim)
    return QWA_ERR_INVALID_ARG;

  // work list on the host, longest key-tile count first (as the context path)
  const int sparse = mode == QWA_MODE_FULL ? 0 : (mode == QWA_MODE_SPARSE ? 1 : max_len <= 8192);
  size_t n_items = 0;
  for (int b = 0; b < batch; ++b) n_items += static_cast<size_t>((cu[b + 1] - cu[b] + kBlockM - 1) / kBlockM) * kKVHeads;
  if (n_items > kMaxItems) return QWA_ERR_INVALID_ARG;  // does not fit the fixed scratch
  std::vector<std::pair<int, AttnItem>> work;
  work.reserve(n_items);
  for (int b = 0; b < batch; ++b) {
    const int len = cu[b + 1] - cu[b];
    for (int q0 = 0; q0 < len; q0 += kBlockM) {
      const int tiles = make_key_schedule(q0, len, sparse, prefix, window).n;
      for (int g = 0; g < kKVHeads; ++g) work.push_back({tiles, make_int4(cu[b] + q0, q0, len, g)});
    }
  }
  std::stable_sort(work.begin(), work.end(),
                   [](const std::pair<int, AttnItem>& a, const std::pair<int, AttnItem>& b) {
                     return a.first > b.first;
                   });
  std::vector<AttnItem> items(work.size());
  for (size_t i = 0; i < work.size(); ++i) items[i] = work[i].second;

  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices)
    return QWA_ERR_CUDA;
  unsigned char* scratch = nullptr;
  qwa_status st = setup_device(device, &scratch);
  if (st != QWA_OK) return st;
  int* status = reinterpret_cast<int*>(scratch);
  AttnItem* d_items = reinterpret_cast<AttnItem*>(scratch + kStatusBytes);

  CUtensorMap tm_q, tm_k, tm_v, tm_o;
  if (!map3d(&tm_q, q, kQHeads, total, kQHeads * kHeadDim * 2) ||
      !map3d(&tm_o, out, kQHeads, total, kQHeads * kHeadDim * 2) ||
      !map3d(&tm_k, k, kKVHeads, total, kKVHeads * kHeadDim * 2) ||
      !map3d(&tm_v, v_base, kKVHeads, total, v_stride * 2))
    return QWA_ERR_CUDA;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // pageable source: the copy is staged before cudaMemcpyAsync returns
  if (cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess ||
      cudaMemcpyAsync(d_items, items.data(), sizeof(AttnItem) * items.size(),
                      cudaMemcpyHostToDevice, s) != cudaSuccess)
    return QWA_ERR_CUDA;
  AttnArgs args;
  args.items = d_items;
  args.out = static_cast<__half*>(out);
  args.sparse = sparse;
  args.prefix = prefix;
  args.window = window;
  args.scale_log2 = 0.08838834764831845f * 1.4426950408889634f;
  args.status = status;
  args.trace = nullptr;
  if (launch_attention(tm_q, tm_k, tm_v, tm_o, args, static_cast<int>(items.size()), s) !=
      cudaSuccess)
    return QWA_ERR_CUDA;
  return QWA_OK;
}
