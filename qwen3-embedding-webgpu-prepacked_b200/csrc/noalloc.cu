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
// holds it until the process exits. A call whose work list does not fit, or
// with more than kMaxBatch requests, is rejected with QWA_ERR_INVALID_ARG
// before anything is launched.
//
// The work list is built on the device by build_items_kernel from the
// call's cu_seqlens, which travel by value in the kernel's parameters: the
// call enqueues two kernels and no host-to-device copy, so nothing it
// enqueues reads host memory after it returns.
//
// The array's name is only a host-side stand-in; the device address is
// obtained once per device with cudaGetSymbolAddress, on the first call made
// with that device current. Make that first call before any stream capture.
// All calls share the one array and it keeps the last call's contents: the
// build kernel clears the status word and rewrites the work list on every
// call, and calls whose launches overlap on the GPU (different streams, no
// ordering between them) race on the work list and produce wrong results.
// A device-side timeout recorded in the status word is reported by
// qwa_check(NULL, stream).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "../../include/qwa.h"
#include "internal.h"

using namespace qwa;

namespace {

constexpr size_t kScratchBytes = 1u << 20;  // 1 MiB
constexpr size_t kStatusBytes = 256;        // status word, padded
constexpr size_t kMaxItems = (kScratchBytes - kStatusBytes) / sizeof(AttnItem);  // 65,520
constexpr int kMaxBatch = 4096;  // cu_seqlens passed by value: 16 KB of kernel parameters
constexpr int kBuildThreads = 1024;
// query tiles of one request at most: every tile is kKVHeads items
constexpr int kMaxQTiles = static_cast<int>(kMaxItems / kKVHeads);

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices] = {};
PFN_cuTensorMapEncodeTiled_v12000 g_encode_na = nullptr;

struct BuildArgs {
  int batch;
  int sparse, prefix, window;
  int max_tiles;  // largest key-tile count of any query tile (histogram size - 1)
  int32_t cu[kMaxBatch + 1];
};

__device__ __forceinline__ int request_of(const BuildArgs& a, const int* tile_off, int t) {
  int lo = 0, hi = a.batch - 1;  // last request whose first query tile is <= t
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tile_off[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// One CTA: clears the status word, then writes the work list sorted by key
// tiles, longest first (a counting sort on the key-tile count; items with
// equal counts may come in any order, which changes no result: every item
// computes its own output tile). Shared memory: tile_off[batch + 1] and
// count[max_tiles + 1].
__global__ void __launch_bounds__(kBuildThreads, 1)
    build_items_kernel(const __grid_constant__ BuildArgs a, AttnItem* items, int* status) {
  extern __shared__ int sh[];
  int* tile_off = sh;                 // [batch + 1]: first query tile of each request
  int* count = sh + (a.batch + 1);    // [max_tiles + 1]: items, then next slot, per count
  __shared__ int total_tiles;
  if (threadIdx.x == 0) {
    *status = 0;
    int acc = 0;
    for (int b = 0; b < a.batch; ++b) {
      tile_off[b] = acc;
      acc += (a.cu[b + 1] - a.cu[b] + kBlockM - 1) / kBlockM;
    }
    tile_off[a.batch] = acc;
    total_tiles = acc;
  }
  for (int i = threadIdx.x; i <= a.max_tiles; i += blockDim.x) count[i] = 0;
  __syncthreads();
  const int nt = total_tiles;
  for (int t = threadIdx.x; t < nt; t += blockDim.x) {
    const int b = request_of(a, tile_off, t);
    const int len = a.cu[b + 1] - a.cu[b];
    const int q0 = (t - tile_off[b]) * kBlockM;
    atomicAdd(&count[make_key_schedule(q0, len, a.sparse, a.prefix, a.window).n], kKVHeads);
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // first slot of each count, largest count first
    int acc = 0;
    for (int n = a.max_tiles; n >= 0; --n) {
      const int c = count[n];
      count[n] = acc;
      acc += c;
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < nt; t += blockDim.x) {
    const int b = request_of(a, tile_off, t);
    const int len = a.cu[b + 1] - a.cu[b];
    const int q0 = (t - tile_off[b]) * kBlockM;
    const int n = make_key_schedule(q0, len, a.sparse, a.prefix, a.window).n;
    const int pos = atomicAdd(&count[n], kKVHeads);
    for (int g = 0; g < kKVHeads; ++g) items[pos + g] = make_int4(a.cu[b] + q0, q0, len, g);
  }
}

qwa_status setup_device(int device, unsigned char** out) {
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
    if (cudaFuncSetAttribute(build_items_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(sizeof(int) * (kMaxBatch + 1 + kMaxQTiles + 2))) !=
        cudaSuccess)
      return QWA_ERR_CUDA;
    g_scratch_ptr[device] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch_ptr[device]);
  return QWA_OK;
}

bool map3d(CUtensorMap* map, const void* base, int heads, int64_t rows, int64_t row_stride,
           uint32_t box_rows = 128) {
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[2] = {256, static_cast<cuuint64_t>(row_stride)};
  cuuint32_t box[3] = {64, 1, box_rows};
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
  if (!cu || batch < 1 || batch > kMaxBatch || cu[0] != 0) return QWA_ERR_INVALID_ARG;
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
  const size_t n_items = count_work_items(cu, batch);
  if (n_items > kMaxItems) return QWA_ERR_INVALID_ARG;  // does not fit the fixed scratch

  BuildArgs a;
  a.batch = batch;
  a.sparse = resolve_sparse(mode, max_len);
  a.prefix = prefix;
  a.window = window;
  // every query tile's key-tile count is at most that of the tile at the same
  // offset in the longest request
  a.max_tiles = 0;
  for (int q0 = 0; q0 < max_len; q0 += kBlockM) {
    const int n = make_key_schedule(q0, max_len, a.sparse, prefix, window).n;
    a.max_tiles = n > a.max_tiles ? n : a.max_tiles;
  }
  for (int b = 0; b <= batch; ++b) a.cu[b] = cu[b];

  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices)
    return QWA_ERR_CUDA;
  // Held from the set-up through both launches, so calls from several host
  // threads on one stream enqueue each call's build and attention together.
  std::lock_guard<std::mutex> lock(g_mutex);
  unsigned char* scratch = nullptr;
  qwa_status st = setup_device(device, &scratch);
  if (st != QWA_OK) return st;
  int* status = reinterpret_cast<int*>(scratch);
  AttnItem* d_items = reinterpret_cast<AttnItem*>(scratch + kStatusBytes);

  CUtensorMap tm_q, tm_k, tm_v, tm_o;
  if (!map3d(&tm_q, q, kQHeads, total, kQHeads * kHeadDim * 2) ||
      !map3d(&tm_o, out, kQHeads, total, kQHeads * kHeadDim * 2, kOutBoxRows) ||
      !map3d(&tm_k, k, kKVHeads, total, kKVHeads * kHeadDim * 2) ||
      !map3d(&tm_v, v_base, kKVHeads, total, v_stride * 2))
    return QWA_ERR_CUDA;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t shmem = sizeof(int) * (batch + 1 + a.max_tiles + 1);
  build_items_kernel<<<1, kBuildThreads, shmem, s>>>(a, d_items, status);
  if (cudaGetLastError() != cudaSuccess) return QWA_ERR_CUDA;
  AttnArgs args;
  args.items = d_items;
  args.out = static_cast<__half*>(out);
  args.sparse = a.sparse;
  args.prefix = prefix;
  args.window = window;
  args.scale_log2 = kScale * kLog2e;
  args.status = status;
  args.trace = nullptr;
  if (launch_attention(tm_q, tm_k, tm_v, tm_o, args, static_cast<int>(n_items), s) !=
      cudaSuccess)
    return QWA_ERR_CUDA;
  return QWA_OK;
}

// Status word of the allocation-free path on the current device (for
// qwa_check(NULL, stream)): synchronises the stream, reads and clears it.
// C linkage to match its declaration in api.cu; not exported (hidden).
extern "C" qwa_status qwa_noalloc_status(void* stream) {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices)
    return QWA_ERR_CUDA;
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return QWA_ERR_CUDA;
  unsigned char* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    scratch = static_cast<unsigned char*>(g_scratch_ptr[device]);
  }
  if (!scratch) return QWA_OK;  // no allocation-free call ran on this device
  int code = 0;
  if (cudaMemcpy(&code, scratch, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return QWA_ERR_CUDA;
  if (code == 0) return QWA_OK;
  if (cudaMemset(scratch, 0, sizeof(int)) != cudaSuccess) return QWA_ERR_CUDA;
  return QWA_ERR_TIMEOUT;
}
