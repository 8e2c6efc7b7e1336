// Causal / sparse GQA prefill attention for sm_100a (tcgen05 + TMA + TMEM).
//
// Replaces the reference's tiledFlashAttentionShader and the chunked two-pass
// path (src/webgpu/ops.ts:168-316): same kept-pair predicate (ops.ts:220),
// fp32 softmax/accumulation instead of the shader's f16 accumulators.
//
// One CTA = one 128-row query tile of one request for BOTH query heads
// (2g, 2g+1) that share key/value head g, so each K/V tile is loaded once for
// two MMA streams (GQA 2:1).
//
// Warp roles (384 threads, three warpgroups):
//   warp 0      TMA producer: Q tiles once, then K_j / V_j into a 3-slot ring
//   warp 1      TMEM owner; lane 0 issues every tcgen05.mma and commit
//   warps 2-3   idle (they complete warpgroup 0, whose registers
//               setmaxnreg lowers to 104 so the softmax warps get 200)
//   warps 4-7   softmax warpgroup A (head 2g):   one thread per query row
//   warps 8-11  softmax warpgroup B (head 2g+1)
//
// TMEM (512 columns x 128 lanes, fp32):
//   [0,128)   S_A = Q_A K_j^T   (P_A, f16 packed, overwrites columns [0,64))
//   [128,256) S_B
//   [256,384) O_A accumulator
//   [384,512) O_B accumulator
//
// MMA issue order per key tile j (in-order tensor pipe):
//   S_A(j), PV_B(j-1), S_B(j), PV_A(j)
// so S_X(j)'s commit also proves PV_X(j-1) finished: the softmax warpgroup
// can then rescale O_X in TMEM, and write P_X(j) over S_X(j), without a
// separate correction warpgroup. Softmax of A overlaps the B MMAs and
// vice versa.
//
// Masked key tiles are never visited: the key-tile schedule enumerates only
// tiles that hold a kept pair (prefix tiles + window tiles in sparse mode);
// elementwise masking runs only on tiles that straddle a mask boundary.
#include <cuda_fp16.h>

#include "attn_common.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace qwa {
namespace {
using namespace attn;

#ifdef QWA_TRACE
// Trace events (clock64): producer K/V issue, MMA issue points, and for row 0
// of each softmax warpgroup the S wait / TMEM load / max / exp / P arrive.
enum TraceEvent : int {
  kTrK = 0, kTrV, kTrMmaSA, kTrMmaPVB, kTrMmaSB, kTrMmaPVA,
  kTrSmSReady, kTrSmLoaded = kTrSmSReady + 2, kTrSmMax = kTrSmLoaded + 2,
  kTrSmExp = kTrSmMax + 2, kTrSmArrive = kTrSmExp + 2, kTrEpi = kTrSmArrive + 2,
  kTrEpiEnd = kTrEpi + 2, kTrMmaPHiA = kTrEpiEnd + 2, kTrMmaKWait, kTrMmaPHiB,
  kTrMmaPVAHiDone, kTrMmaSADone,
  kTrWarpMax,             // +softmax warp (0..7): lane 0 after the row max
  kTrWarpArrive = kTrWarpMax + 8,   // +softmax warp: lane 0 at its P-hi arrival
  kTrEpiChunk = kTrWarpArrive + 8,  // CTA entry/exit: [0]/[1] globaltimer, [2]/[3] clock64
  kTrEpiStaged = kTrEpiChunk + 8,   // issuer: +0 before / +1 after its Q wait (first tile t)
  kTrEpiIssued = kTrEpiStaged + 2,  // producer: +0 Q load issued (item li)
  kTrWarpEpi = kTrEpiIssued + 2,    // +softmax warp: lane 0 past the O-final wait
  kTrWarpStaged = kTrWarpEpi + 8    // +softmax warp: lane 0 at its staged arrival
};
#define QWA_TR(ev, j)                                                                \
  do {                                                                               \
    if (args.trace && blockIdx.x < kTraceCtas && (j) < kTraceIters)                  \
      args.trace[(blockIdx.x * kTraceEvents + (ev)) * kTraceIters + (j)] = clock64(); \
  } while (0)
#else
#define QWA_TR(ev, j) \
  do {                \
  } while (0)
#endif

// Warpgroup 0: producer, MMA issuer, two idle warps; warpgroups 1 and 2: the
// softmax of heads A and B. setmaxnreg moves registers from warpgroup 0 to
// the softmax warps (launch: 384 x 168 = 128 x 104 + 256 x 200).
constexpr int kThreads = 384;
constexpr int kSoftmaxWarp0 = 4;
constexpr int kRegsSupport = 104;
constexpr int kRegsSoftmax = 200;
static_assert(128 * kRegsSupport + 256 * kRegsSoftmax <= kThreads * 168, "register split");
constexpr uint32_t kQEmptyArrivals = 8;  // every softmax warp stores its own rows
constexpr int kSlots = 3;  // K/V ring (K_j and V_j alternate)
constexpr uint32_t kQOff = 0;  // two Q buffers, each Q_A then Q_B
constexpr uint32_t kQBufBytes = 2 * kTileBytes;
constexpr uint32_t kSlotOff = 2 * kQBufBytes;
constexpr uint32_t kBarOff = kSlotOff + kSlots * kTileBytes;  // 229376
enum Bar : int {
  kQFull = 0,                        // +Q buffer
  kQEmpty = kQFull + 2,              // +Q buffer
  kSlotFull = kQEmpty + 2,           // +slot
  kSlotEmpty = kSlotFull + kSlots,   // +slot
  kSFull = kSlotEmpty + kSlots,      // +X
  kPLo = kSFull + 2,                 // +X: P of keys 0..63 in TMEM
  kPHi = kPLo + 2,                   // +X: P of keys 64..127 in TMEM
  kOFinal = kPHi + 2,              // +X: O_X of the item complete
  kDrain = kOFinal + 2,              // the issuer's MMAs all complete (at exit)
  kNumBars = kDrain + 1
};
constexpr uint32_t kHolderOff = kBarOff + 8 * kNumBars;
constexpr uint32_t kAbortOff = kHolderOff + 4;
constexpr uint32_t kLimitOff = kHolderOff + 8;  // bounded-wait limit (ns), 8-byte aligned
static_assert(kLimitOff % 8 == 0, "limit alignment");
constexpr uint32_t kSmemUsed = kLimitOff + 8;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024;  // + alignment slack
static_assert(kSmemBytes <= 232448, "shared memory budget");

__global__ void __launch_bounds__(kThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ CUtensorMap tm_o, const AttnArgs args,
                     int num_items) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_addr(smem);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kHolderOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kAbortOff);
  volatile unsigned long long* wait_limit =
      reinterpret_cast<volatile unsigned long long*>(smem + kLimitOff);
  auto bar = [&](int i) -> uint32_t { return sbase + kBarOff + 8u * i; };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int sparse = args.sparse, prefix = args.prefix, window = args.window;

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(kQFull + b), 1);
      mbar_init(bar(kQEmpty + b), kQEmptyArrivals);  // one arrival per softmax warp
    }
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(bar(kSlotFull + s), 1);
      mbar_init(bar(kSlotEmpty + s), 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(bar(kSFull + x), 1);
      mbar_init(bar(kPLo + x), 128);
      mbar_init(bar(kPHi + x), 128);
    }
    for (int x = 0; x < 2; ++x) mbar_init(bar(kOFinal + x), 1);
    mbar_init(bar(kDrain), 1);
    *abort_flag = 0;
    *wait_limit = args.wait_ns;
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_o);
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_holder), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
#ifdef QWA_TRACE
  if (threadIdx.x == 0 && args.trace && blockIdx.x < kTraceCtas) {
    args.trace[(blockIdx.x * kTraceEvents + kTrEpiChunk) * kTraceIters + 0] = globaltimer();
    args.trace[(blockIdx.x * kTraceEvents + kTrEpiChunk) * kTraceIters + 2] = clock64();
  }
#endif

  // Work items of this CTA: its own list from the plan's schedule (longest
  // first), or blockIdx.x, blockIdx.x + gridDim.x, ... without one. li counts
  // this CTA's items, t its key tiles across items; every role walks the same
  // sequence, so barrier phases follow from li and t.
  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsSupport));
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int c = 0;  // K/V ring uses
      bool ok = true;
      // last full phase issued per K/V slot (bits 0-2) and Q buffer (bits
      // 3-4): bit i+8 set once one was issued, bit i its parity. Waited for
      // before exit so no copy lands after it.
      uint32_t issued = 0;
      const ItemRange rng = item_range(args, num_items);
      AttnItem next_item = rng.beg < rng.end ? args.items[rng.beg] : AttnItem{};
      for (int it = rng.beg, li = 0; ok && it < rng.end; it += rng.stride, ++li) {
        // the next item's descriptor is loaded one item ahead (a global load
        // at every item boundary sat on each role's critical path)
        const AttnItem item = next_item;
        if (it + rng.stride < rng.end) next_item = args.items[it + rng.stride];
        const int row0 = item.x, q0 = item.y, len = item.z, g = item.w;
        const KeySchedule sch = make_key_schedule(q0, len, sparse, prefix, window);
        const int qb = li & 1;
        if (!(ok = mbar_wait(bar(kQEmpty + qb), ((li >> 1) & 1) ^ 1, abort_flag, args.status,
                             kDevTimeoutQ, wait_limit)))
          break;
        QWA_TR(kTrEpiIssued + 0, li);
        mbar_arrive_expect_tx(bar(kQFull + qb), kQBufBytes);
        issued = (issued & ~(1u << (kSlots + qb))) | (1u << (kSlots + qb + 8)) |
                 (static_cast<uint32_t>((li >> 1) & 1) << (kSlots + qb));
        for (int x = 0; x < 2; ++x) {
          const uint32_t dst = sbase + kQOff + qb * kQBufBytes + x * kTileBytes;
          tma_load_3d(dst, &tm_q, bar(kQFull + qb), 0, 2 * g + x, row0);
          tma_load_3d(dst + kHalfBytes, &tm_q, bar(kQFull + qb), 64, 2 * g + x, row0);
        }
        for (int j = 0; ok && j < sch.n; ++j) {
          const int krow = row0 - q0 + key_tile_start(sch, j);
          for (int kv = 0; kv < 2; ++kv, ++c) {
            const int s = c % kSlots;
            if (!(ok = mbar_wait(bar(kSlotEmpty + s), ((c / kSlots) & 1) ^ 1, abort_flag,
                                 args.status, kDevTimeoutSlotEmpty, wait_limit)))
              break;
            // test hook (qwa_set_debug): CTA 0 leaves one load out, so the
            // MMA issuer's bounded wait for it runs out
            if (blockIdx.x == 0 && c == args.skip_load) continue;
            const uint32_t dst = sbase + kSlotOff + s * kTileBytes;
            const CUtensorMap* tm = kv == 0 ? &tm_k : &tm_v;
            mbar_arrive_expect_tx(bar(kSlotFull + s), kTileBytes);
            issued = (issued & ~(1u << s)) | (1u << (s + 8)) |
                     (static_cast<uint32_t>((c / kSlots) & 1) << s);
            QWA_TR(kTrK + kv, c >> 1);
            tma_load_3d(dst, tm, bar(kSlotFull + s), 0, g, krow);
            tma_load_3d(dst + kHalfBytes, tm, bar(kSlotFull + s), 64, g, krow);
          }
        }
      }
      // Every issued copy has landed before the CTA exits (after an abort some
      // were never consumed). At most one phase per slot or buffer is in
      // flight, so the last issued parity identifies it.
      bool drained = true;
      for (int i = 0; i < kSlots + 2; ++i)
        if ((issued >> (i + 8)) & 1u)
          drained &= mbar_drain(i < kSlots ? bar(kSlotFull + i) : bar(kQFull + i - kSlots),
                                (issued >> i) & 1u, *wait_limit);
      if (!drained) atomicCAS(args.status, 0, kDevTimeoutDrain);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    // One flat stream over all key tiles of all items:
    //   S_A(t), PV_B(t-1), S_B(t), PV_A(t)
    // (the in-order tensor pipe then guarantees S_X(t+1) overwrites P_X(t)
    // only after PV_X(t) read it). PV_B of an item's last tile is issued after
    // the next item's S_A(0), so the next item's MMAs overlap this item's
    // final softmax and epilogue.
    if (lane == 0) {
      const uint32_t t_s[2] = {tmem, tmem + 128};
      const uint32_t t_o[2] = {tmem + 256, tmem + 384};
      const uint64_t q_desc0 = smem_desc_sw128(sbase + kQOff, 16, 1024);
      // slot s's descriptors = slot 0's + (s * kTileBytes) >> 4
      const uint64_t k_desc0 = smem_desc_sw128(sbase + kSlotOff, 16, 1024);
      const uint64_t v_desc0 = smem_desc_sw128(sbase + kSlotOff, kHalfBytes, 1024);
      bool ok = true;
      int t = 0;
      bool have_prev = false;  // PV_B of the previous tile still to issue
      int prev_v = 0, prev_j = 0, prev_nk = 8;
      bool prev_last = false;
      const ItemRange rng = item_range(args, num_items);
      AttnItem next_item = rng.beg < rng.end ? args.items[rng.beg] : AttnItem{};
      for (int it = rng.beg, li = 0; ok && it < rng.end; it += rng.stride, ++li) {
        // the next item's descriptor is loaded one item ahead (a global load
        // at every item boundary sat on each role's critical path)
        const AttnItem item = next_item;
        if (it + rng.stride < rng.end) next_item = args.items[it + rng.stride];
        const KeySchedule sch = make_key_schedule(item.y, item.z, sparse, prefix, window);
        const int q_last = (item.y + kBlockM < item.z ? item.y + kBlockM : item.z) - 1;
        const int qb = li & 1;
        const uint64_t qa = q_desc0 + ((qb * kQBufBytes) >> 4);
        const uint64_t qbd = qa + (kTileBytes >> 4);
        QWA_TR(kTrEpiStaged + 0, t);
        if (!(ok = mbar_wait(bar(kQFull + qb), (li >> 1) & 1, abort_flag, args.status,
                             kDevTimeoutQ, wait_limit)))
          break;
        QWA_TR(kTrEpiStaged + 1, t);
        for (int j = 0; j < sch.n; ++j, ++t) {
          const int ck = 2 * t, sk = ck % kSlots;
          const int cv = 2 * t + 1, sv = cv % kSlots;
          const uint64_t k_desc = k_desc0 + ((sk * kTileBytes) >> 4);
          QWA_TR(kTrMmaKWait, t);
          if (!(ok = mbar_wait(bar(kSlotFull + sk), (ck / kSlots) & 1, abort_flag, args.status,
                               kDevTimeoutSlotFull, wait_limit)))
            break;
          tc_fence_after();
          QWA_TR(kTrMmaSA, t);
          const int width = key_tile_width(sch, j, q_last, prefix);
          const uint32_t idesc = idesc_f16_f32(128, width, false);
          issue_qk(t_s[0], qa, k_desc, idesc);
          QWA_TR(kTrMmaSADone, t);
          tc_commit(bar(kSFull + 0));
          if (have_prev) {
            const uint64_t vd = v_desc0 + ((prev_v * kTileBytes) >> 4);
            if (!(ok = mbar_wait(bar(kPLo + 1), (t - 1) & 1, abort_flag, args.status,
                                 kDevTimeoutPFull, wait_limit)))
              break;
            tc_fence_after();
            QWA_TR(kTrMmaPVB, t - 1);
            issue_pv_half(t_o[1], t_s[1], vd, prev_j > 0, prev_nk, 0);
            if (!(ok = mbar_wait(bar(kPHi + 1), (t - 1) & 1, abort_flag, args.status,
                                 kDevTimeoutPFull, wait_limit)))
              break;
            tc_fence_after();
            QWA_TR(kTrMmaPHiB, t - 1);
            issue_pv_half(t_o[1], t_s[1], vd, prev_j > 0, prev_nk, 1);
            tc_commit(bar(kSlotEmpty + prev_v));
            if (prev_last) tc_commit(bar(kOFinal + 1));
          }
          QWA_TR(kTrMmaSB, t);
          issue_qk(t_s[1], qbd, k_desc, idesc);
          tc_commit(bar(kSFull + 1));
          tc_commit(bar(kSlotEmpty + sk));
          if (!(ok = mbar_wait(bar(kSlotFull + sv), (cv / kSlots) & 1, abort_flag, args.status,
                               kDevTimeoutSlotFull, wait_limit)))
            break;
          {
            const uint64_t vd = v_desc0 + ((sv * kTileBytes) >> 4);
            if (!(ok = mbar_wait(bar(kPLo + 0), t & 1, abort_flag, args.status,
                                 kDevTimeoutPFull, wait_limit)))
              break;
            tc_fence_after();
            QWA_TR(kTrMmaPVA, t);
            issue_pv_half(t_o[0], t_s[0], vd, j > 0, width / 16, 0);
            if (!(ok = mbar_wait(bar(kPHi + 0), t & 1, abort_flag, args.status,
                                 kDevTimeoutPFull, wait_limit)))
              break;
            tc_fence_after();
            QWA_TR(kTrMmaPHiA, t);
            issue_pv_half(t_o[0], t_s[0], vd, j > 0, width / 16, 1);
            QWA_TR(kTrMmaPVAHiDone, t);
          }
          // head A's output is final here; its epilogue need not wait for B
          if (j == sch.n - 1) tc_commit(bar(kOFinal + 0));
          have_prev = true;
          prev_v = sv;
          prev_j = j;
          prev_nk = width / 16;
          prev_last = j == sch.n - 1;
        }
      }
      if (ok && have_prev &&
          mbar_wait(bar(kPLo + 1), (t - 1) & 1, abort_flag, args.status, kDevTimeoutPFull, wait_limit)) {
        const uint64_t vd = v_desc0 + ((prev_v * kTileBytes) >> 4);
        tc_fence_after();
        issue_pv_half(t_o[1], t_s[1], vd, prev_j > 0, prev_nk, 0);
        if (mbar_wait(bar(kPHi + 1), (t - 1) & 1, abort_flag, args.status, kDevTimeoutPFull, wait_limit)) {
          tc_fence_after();
          issue_pv_half(t_o[1], t_s[1], vd, prev_j > 0, prev_nk, 1);
          tc_commit(bar(kSlotEmpty + prev_v));
          tc_commit(bar(kOFinal + 1));
        }
      }
      // Every issued MMA has completed before TMEM is released (after an abort
      // nothing else waits for them).
      tc_commit(bar(kDrain));
      if (!mbar_drain(bar(kDrain), 0, *wait_limit)) atomicCAS(args.status, 0, kDevTimeoutDrain);
    }
  }
  } else {
    // softmax warpgroups take the registers the producer/issuer warpgroup gave up
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    // ------------------------------------------------------------- softmax
    const int x = (warp - kSoftmaxWarp0) >> 2;  // 0: head 2g, 1: head 2g+1
    const int sub = warp & 3;       // TMEM lane sub-partition of this warp
    const int row = sub * 32 + lane;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(sub * 32) << 16);
    const uint32_t t_s = t_lane + x * 128;
    const uint32_t t_o = t_lane + 256 + x * 128;
    const float scale = args.scale_log2;
    bool ok = true;
    int t = 0;
    int q_release = -1;  // lane 0: Q buffer to release once its O stores read it
    const ItemRange rng = item_range(args, num_items);
    AttnItem next_item = rng.beg < rng.end ? args.items[rng.beg] : AttnItem{};
    for (int it = rng.beg, li = 0; ok && it < rng.end; it += rng.stride, ++li) {
      const AttnItem item = next_item;
      if (it + rng.stride < rng.end) next_item = args.items[it + rng.stride];
      const int row0 = item.x, q0 = item.y, len = item.z, g = item.w;
      const KeySchedule sch = make_key_schedule(q0, len, sparse, prefix, window);
      const int q = q0 + row;
      const int q_last = (q0 + kBlockM < len ? q0 + kBlockM : len) - 1;
      float m_run = -INFINITY;  // running max of scaled scores (log2 domain)
      float l_run = 0.f;        // running denominator relative to m_run
      for (int j = 0; j < sch.n; ++j, ++t) {
        if (!(ok = mbar_wait(bar(kSFull + x), t & 1, abort_flag, args.status, kDevTimeoutSFull, wait_limit)))
          break;
        tc_fence_after();
        if (row == 0) QWA_TR(kTrSmSReady + x, t);
        const int ks = key_tile_start(sch, j);
        // narrow tile (width <= 64): only its first two 32-column chunks exist;
        // columns past the width are stale TMEM and always masked below
        const bool narrow = key_tile_width(sch, j, q_last, prefix) <= 64;
        uint32_t a0[32], a1[32], a2[32], a3[32];
        tmem_ld32(t_s + 0, a0);
        tmem_ld32(t_s + 32, a1);
        if (!narrow) {
          tmem_ld32(t_s + 64, a2);
          tmem_ld32(t_s + 96, a3);
        }
        tmem_wait_ld();
        reg_fence32(a0);
        reg_fence32(a1);
        if (!narrow) {
          reg_fence32(a2);
          reg_fence32(a3);
        }
        if (row == 0) QWA_TR(kTrSmLoaded + x, t);
        if (tile_needs_mask(sch, j, ks, q0, q_last, sparse, prefix, window)) {
          const int kcap = (sch.split && j < sch.n_prefix) ? prefix : 0x7fffffff;
          mask_chunk(a0, ks + 0, q, kcap, sparse, prefix, window);
          mask_chunk(a1, ks + 32, q, kcap, sparse, prefix, window);
          if (!narrow) {
            mask_chunk(a2, ks + 64, q, kcap, sparse, prefix, window);
            mask_chunk(a3, ks + 96, q, kcap, sparse, prefix, window);
          }
        }
        // Raw scores; the softmax scale is folded into the exponent below.
        float tmax = fmaxf(chunk_max(a0), chunk_max(a1));
        if (!narrow) tmax = fmaxf(tmax, fmaxf(chunk_max(a2), chunk_max(a3)));
        tmax *= scale;
        const float m_new = fmaxf(m_run, tmax);
        bool need = false;
        float f = 1.f;
        if (j == 0) {
          m_run = m_new;
        } else if (m_new > m_run + 8.f) {
          // Lazy rescale: keep the stale max unless the new one exceeds it by
          // more than 2^8 (P stays <= 256, exact enough in f16 and fp32).
          need = true;
          f = ex2(m_run - m_new);
          l_run *= f;
          m_run = m_new;
        }
        if (row == 0) QWA_TR(kTrSmMax + x, t);
        if (lane == 0) QWA_TR(kTrWarpMax + warp - kSoftmaxWarp0, t);
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        // P is published in two halves so PV's first four K steps (keys
        // 0..63) run on the tensor pipe while keys 64..127 are exponentiated.
        float sum = exp_pack_chunk(a0, scale, m_use) + exp_pack_chunk(a1, scale, m_use);
        tmem_st16(t_s + 0, a0);
        tmem_st16(t_s + 16, a1);
        if (__any_sync(0xffffffffu, need)) {
          // O_X(j-1) is complete (S_X(j) was committed after PV_X(j-1)); the
          // rescale precedes the first P arrival, so no PV_X(j) step sees it
          // half done.
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(t_o + 32 * c, o);
            tmem_wait_ld();
            reg_fence32(o);
            const uint64_t f2 = f2_pack(f, f);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float r0, r1;
              f2_unpack(mul2(f2_pack(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1])), f2),
                        r0, r1);
              o[2 * i] = __float_as_uint(r0);
              o[2 * i + 1] = __float_as_uint(r1);
            }
            tmem_st32(t_o + 32 * c, o);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar(kPLo + x));
        if (!narrow) {
          sum += exp_pack_chunk(a2, scale, m_use) + exp_pack_chunk(a3, scale, m_use);
          tmem_st16(t_s + 32, a2);
          tmem_st16(t_s + 48, a3);
          tmem_wait_st();
          tc_fence_before();
        }
        l_run += sum;
        if (row == 0) QWA_TR(kTrSmExp + x, t);
        mbar_arrive(bar(kPHi + x));
        if (row == 0) QWA_TR(kTrSmArrive + x, t);
        if (lane == 0) QWA_TR(kTrWarpArrive + warp - kSoftmaxWarp0, t);
        if (q_release >= 0) {  // storing threads only: see the epilogue
          bulk_wait_read();
          mbar_arrive(bar(kQEmpty + q_release));
          q_release = -1;
        }
      }
      // Epilogue. O_X is read to registers (wait::ld) before this warpgroup's
      // next P arrival, which is what the next item's first PV_X waits for.
      if (!ok || !(ok = mbar_wait(bar(kOFinal + x), li & 1, abort_flag, args.status,
                                  kDevTimeoutOFinal, wait_limit)))
        break;
      tc_fence_after();
      if (row == 0) QWA_TR(kTrEpi + x, t - 1);
      if (lane == 0) QWA_TR(kTrWarpEpi + warp - kSoftmaxWarp0, t - 1);
      const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
      const int qb = li & 1;
      if (q0 + kBlockM <= len) {
        // Full query tile: O goes through this item's Q buffer (free: the
        // last S MMAs that read it completed before kOFinal) in the 128-byte
        // swizzled layout Q arrived in, then out with two TMA stores per head.
        // The warp-wide direct stores this replaces touched 32 rows 4 KB apart
        // per instruction.
        const uint32_t obuf = sbase + kQOff + qb * kQBufBytes + x * kTileBytes;
        // Each warp stages its own 32 rows and stores them with two TMA
        // stores (boxes of 32 rows): no barrier across the warpgroup on the
        // way to the next item. (A warpgroup-wide staged barrier with one
        // storing thread measured 2-9% slower on short requests.)
        {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(t_o + 32 * c, o);
            tmem_wait_ld();
            reg_fence32(o);
            const uint32_t half_base = obuf + (c >> 1) * kHalfBytes + row * 128;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const uint32_t unit = static_cast<uint32_t>((c & 1) * 4 + v) ^ (row & 7);
              const uint32_t* p = o + 8 * v;
              const uint32_t w0 = pack_half2(__uint_as_float(p[0]) * inv_l, __uint_as_float(p[1]) * inv_l);
              const uint32_t w1 = pack_half2(__uint_as_float(p[2]) * inv_l, __uint_as_float(p[3]) * inv_l);
              const uint32_t w2 = pack_half2(__uint_as_float(p[4]) * inv_l, __uint_as_float(p[5]) * inv_l);
              const uint32_t w3 = pack_half2(__uint_as_float(p[6]) * inv_l, __uint_as_float(p[7]) * inv_l);
              asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(half_base + unit * 16),
                           "r"(w0), "r"(w1), "r"(w2), "r"(w3)
                           : "memory");
            }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          QWA_TR(kTrWarpStaged + warp - kSoftmaxWarp0, t - 1);
          const uint32_t rows_off = static_cast<uint32_t>(sub * 32 * 128);
          tma_store_3d(&tm_o, obuf + rows_off, 0, 2 * g + x, row0 + sub * 32);
          tma_store_3d(&tm_o, obuf + kHalfBytes + rows_off, 64, 2 * g + x, row0 + sub * 32);
          bulk_commit();
          // released after this head's next P arrival, once the stores read it
          q_release = qb;
        }
      } else {
        // Last, partial tile of a request: rows past len belong to the next
        // request, so only valid rows are stored, directly.
        const bool valid = q < len;
        __half* dst = args.out + (static_cast<int64_t>(row0 + row) * kQHeads + 2 * g + x) * kHeadDim;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(t_o + 32 * c, o);
          tmem_wait_ld();
          reg_fence32(o);
          if (valid) {
            uint4* d4 = reinterpret_cast<uint4*>(dst + 32 * c);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 w;
              w.x = pack_half2(__uint_as_float(o[8 * v + 0]) * inv_l, __uint_as_float(o[8 * v + 1]) * inv_l);
              w.y = pack_half2(__uint_as_float(o[8 * v + 2]) * inv_l, __uint_as_float(o[8 * v + 3]) * inv_l);
              w.z = pack_half2(__uint_as_float(o[8 * v + 4]) * inv_l, __uint_as_float(o[8 * v + 5]) * inv_l);
              w.w = pack_half2(__uint_as_float(o[8 * v + 6]) * inv_l, __uint_as_float(o[8 * v + 7]) * inv_l);
              d4[v] = w;
            }
          }
        }
        if (lane == 0) mbar_arrive(bar(kQEmpty + qb));
      }
      if (row == 0) QWA_TR(kTrEpiEnd + x, t - 1);
      tc_fence_before();
    }
    if (q_release >= 0) {
      bulk_wait_read();
      mbar_arrive(bar(kQEmpty + q_release));
    }
  }

  bulk_wait_all();  // epilogue stores of the last items (no-op for other threads)
  tc_fence_before();
  __syncthreads();
#ifdef QWA_TRACE
  if (threadIdx.x == 0 && args.trace && blockIdx.x < kTraceCtas) {
    args.trace[(blockIdx.x * kTraceEvents + kTrEpiChunk) * kTraceIters + 1] = globaltimer();
    args.trace[(blockIdx.x * kTraceEvents + kTrEpiChunk) * kTraceIters + 3] = clock64();
  }
#endif
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------- self test
// One S tile and one PV tile through the same descriptors as the kernel above.
__global__ void __launch_bounds__(128, 1)
    selftest_tile_kernel(const __grid_constant__ CUtensorMap tm_a,
                         const __grid_constant__ CUtensorMap tm_b,
                         const __grid_constant__ CUtensorMap tm_v, float* c_out, float* d_out,
                         int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_addr(smem);
  const uint32_t bar_ld = sbase + 3 * kTileBytes, bar_mma = bar_ld + 8;
  uint32_t* holder = reinterpret_cast<uint32_t*>(smem + 3 * kTileBytes + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 3 * kTileBytes + 20);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(bar_ld, 1);
    mbar_init(bar_mma, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_addr(holder), 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *holder;
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(bar_ld, 3 * kTileBytes);
    const CUtensorMap* maps[3] = {&tm_a, &tm_b, &tm_v};
    for (int i = 0; i < 3; ++i) {
      tma_load_3d(sbase + i * kTileBytes, maps[i], bar_ld, 0, 0, 0);
      tma_load_3d(sbase + i * kTileBytes + kHalfBytes, maps[i], bar_ld, 64, 0, 0);
    }
    if (mbar_wait(bar_ld, 0, abort_flag, status, kDevTimeoutSlotFull)) {
      tc_fence_after();
      issue_qk(tmem, smem_desc_sw128(sbase, 16, 1024), smem_desc_sw128(sbase + kTileBytes, 16, 1024));
      tc_commit(bar_mma);
    }
  }
  const uint32_t t_lane = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  const int row = warp * 32 + lane;
  bool ok = mbar_wait(bar_mma, 0, abort_flag, status, kDevTimeoutSFull);
  if (ok) {
    tc_fence_after();
    uint32_t p[2][32];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t r[32];
      tmem_ld32(t_lane + 32 * c, r);
      tmem_wait_ld();
      reg_fence32(r);
#pragma unroll
      for (int i = 0; i < 32; ++i) c_out[row * 128 + 32 * c + i] = __uint_as_float(r[i]);
#pragma unroll
      for (int i = 0; i < 16; ++i)
        p[c >> 1][(c & 1) * 16 + i] = pack_half2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
    }
    tmem_st32(t_lane, p[0]);
    tmem_st32(t_lane + 32, p[1]);
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (ok && threadIdx.x == 0) {
    issue_pv(tmem + 128, tmem, smem_desc_sw128(sbase + 2 * kTileBytes, kHalfBytes, 1024), false);
    tc_commit(bar_mma);
  }
  if (ok && mbar_wait(bar_mma, 1, abort_flag, status, kDevTimeoutOFinal)) {
    tc_fence_after();
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t r[32];
      tmem_ld32(t_lane + 128 + 32 * c, r);
      tmem_wait_ld();
      reg_fence32(r);
#pragma unroll
      for (int i = 0; i < 32; ++i) d_out[row * 128 + 32 * c + i] = __uint_as_float(r[i]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace

cudaError_t launch_attention(const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                             const CUtensorMap& tm_v, const CUtensorMap& tm_o,
                             const AttnArgs& args, int num_items,
                             cudaStream_t stream) {
  // function attributes and SM counts are per device
  static bool configured[kMaxDevices] = {};
  static int sms[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemBytes);
    if (e == cudaSuccess)
      e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  if (num_items <= 0) return cudaSuccess;
  const int sm_count = sms[dev];
  // persistent: one CTA per SM, or the plan's per-CTA item lists
  const int grid = args.cta_offsets ? args.num_ctas
                                    : (num_items < sm_count ? num_items : sm_count);
  attention_kernel<<<grid, kThreads, kSmemBytes, stream>>>(tm_q, tm_k, tm_v, tm_o, args,
                                                           num_items);
  return cudaGetLastError();
}

cudaError_t launch_selftest_tile(const CUtensorMap& tm_a, const CUtensorMap& tm_b,
                                 const CUtensorMap& tm_v, float* c, float* d, int* status,
                                 cudaStream_t stream) {
  const uint32_t bytes = 3 * kTileBytes + 64 + 1024;
  cudaError_t e = cudaFuncSetAttribute(selftest_tile_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  selftest_tile_kernel<<<1, 128, bytes, stream>>>(tm_a, tm_b, tm_v, c, d, status);
  return cudaGetLastError();
}

}  // namespace qwa
