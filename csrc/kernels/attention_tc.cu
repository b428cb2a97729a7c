// PrefixLM packed-varlen flash attention forward on 5th-generation tensor cores (tcgen05).
//
// Same contract as attn_fwd in attention.cu (mask: key j visible to query i of a document
// with prefix P iff j < max(P, i + 1); O, Y = sigmoid(gate) * O and a log2-domain LSE per
// (head, token); zero rows for padding), same device-built work schedule (LPT-ordered
// 128-query tiles, layout: 8 header ints then int4 {doc_start, len, prefix, q0} tiles).
//
// One CTA = one 128-query tile of one head at a time; persistent CTAs pull tiles of the
// LPT-sorted list from a global counter (ItemRing below). Warp roles (320 threads):
//   warp 0      TMA loads: Q tile once, K and V blocks of 128 keys through 2-stage rings
//               (128B-swizzled [128 rows][64] boxes straight from the fused gqkv buffer)
//   warp 1      UMMA issue (one lane): S_j = Q K_j^T into one of two TMEM S buffers, then
//               O_a += P_{j-1}[:, 0:64] V_{j-1}[0:64] and O_b += P_{j-1}[:, 64:128] V_{j-1}[64:128]
//               with P read straight from TMEM (A operand in tensor memory), so S_j runs on
//               the tensor cores while the softmax warps turn S_{j-1} into P_{j-1}
//   warps 2..5  softmax of key half 0 of every block, warps 6..9 of key half 1: one query row
//   and 6..9    per thread (TMEM lane quarter = warp % 4), 64 scores read from TMEM once into
//               registers. Each half keeps its own running max / sum and its own O
//               accumulator, so the two warpgroups never synchronise inside the key loop;
//               the two partial results are merged once per tile in the epilogue (the usual
//               split-softmax combine). A half rescales its O accumulator in TMEM only when
//               its row max grows by more than 8 (log2 units) -- exact, since O and l share
//               the stale max. Two softmax warps per scheduler hide the TMEM/MUFU latency that
//               one warp per scheduler cannot.
// P stays in TMEM: a softmax half writes its 64 probabilities of block j as bf16 pairs into
// the first 32 columns of its own 64-column half of block j's S buffer (the columns it has
// just read), and the PV UMMA reads them from there. P_j and P_{j-1} thus live in different
// buffers, so the softmax of block j never waits for PV_{j-1} (only an O rescale does), and
// S_{j+2} may overwrite buffer j&1 as soon as PV_j has been issued: UMMAs of one thread run in
// issue order.
// Tile turnaround: Q is double-buffered (the next tile's Q arrives while this tile computes),
// the producer passes each work item's tile descriptor through the shared-memory ring (no
// role re-reads the schedule from global memory), and the softmax warps fetch their rows'
// gate values into registers when a tile starts, so the epilogue does no global loads.
// TMEM: S0/P0 [0,128), S1/P1 [128,256), O_a [256,384), O_b [384,512) (the whole 512 columns).
// Shared memory: Q 2 x 32 KB, K 2 x 32 KB, V 2 x 32 KB, per-row (max, sum) exchange 2 KB.
//
// Every mbarrier wait is bounded; on a timeout the CTA records an error, drains its own
// copies and UMMAs, frees TMEM and returns.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "device_setup.h"

namespace hrm {
namespace attn_tc {

constexpr int D = 128, BQ = 128, BKV = 128;
constexpr int SCHED_HEADER = 8;
constexpr int THREADS = 320;
constexpr int TILE_BYTES = 128 * 128 * 2;  // one [128][128] bf16 tile = two [128][64] swizzled boxes
constexpr int ML_BYTES = 2 * 128 * 8;      // per key half and row: (max, sum)
constexpr int SMEM_BYTES = 1024 + 6 * TILE_BYTES + ML_BYTES + 512;
constexpr uint32_t TM_S0 = 0, TM_S1 = 128, TM_OA = 256, TM_OB = 384, TM_COLS = 512;
constexpr float kRescaleThreshold = 8.0f;

// mbarrier wait whose outcome is the same for every lane of the warp (the softmax warps run
// warp-collective TMEM instructions after their waits and must not diverge on a timeout).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

// Dynamic work distribution: the producer warp of each CTA pulls the next item of the
// LPT-ordered list from a global counter and publishes it through a small shared-memory ring;
// every other role of the CTA reads the same sequence. Greedy pulling over a cost-sorted list
// keeps the CTAs' finishing times within about one item of each other (a static stride does
// not: the most expensive items of every round land on the same CTAs).
constexpr int kItemRing = 4;
struct ItemRing {
  uint64_t full[kItemRing], empty[kItemRing];
  int item[kItemRing];
};
__device__ __forceinline__ void ring_init(ItemRing* r, int consumers) {
  for (int i = 0; i < kItemRing; ++i) {
    mbar_init(&r->full[i], 1);
    mbar_init(&r->empty[i], consumers);
  }
}
// producer (one thread): the k-th item of this CTA; false on a wait timeout
__device__ __forceinline__ bool ring_push(ItemRing* r, int k, int* counter, int& item) {
  const int s = k % kItemRing;
  if (!mbar_wait(&r->empty[s], ((k / kItemRing) & 1) ^ 1)) return false;
  item = atomicAdd(counter, 1);
  *reinterpret_cast<volatile int*>(&r->item[s]) = item;
  mbar_arrive(&r->full[s]);  // release: the slot's value is visible to the waiters
  return true;
}
// consumer, one thread; INT_MAX on a wait timeout
__device__ __forceinline__ int ring_pop_thread(ItemRing* r, int k) {
  const int s = k % kItemRing;
  if (!mbar_wait(&r->full[s], (k / kItemRing) & 1)) return INT_MAX;
  const int it = *reinterpret_cast<volatile int*>(&r->item[s]);
  mbar_arrive(&r->empty[s]);
  return it;
}
// consumer, whole warp (same value in every lane); INT_MAX on a wait timeout
__device__ __forceinline__ int ring_pop_warp(ItemRing* r, int k) {
  const int s = k % kItemRing;
  if (!__all_sync(0xffffffffu, mbar_wait(&r->full[s], (k / kItemRing) & 1))) return INT_MAX;
  const int it = *reinterpret_cast<volatile int*>(&r->item[s]);
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&r->empty[s]);
  return it;
}
// last CTA to finish resets the work counters, so one schedule serves every launch
__device__ __forceinline__ void finish_items(int* counter, int* done) {
  __threadfence();
  if (atomicAdd(done, 1) == (int)gridDim.x - 1) {
    *counter = 0;
    *done = 0;
    __threadfence();
  }
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16,"
      " %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  tmem_ld_32x32b_x32(taddr, r);
  tmem_ld_wait();
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

struct Params {
  __nv_bfloat16* out;
  __nv_bfloat16* y;
  const __nv_bfloat16* qkv;  // for the gate
  long ld_out, ld_qkv;
  float* lse;
  int T, H;
  float scale_log2;
  const int* sched;
  int* err;
};

// The forward's ring also carries each item's tile descriptor (read once, by the producer).
struct TileRing {
  uint64_t full[kItemRing], empty[kItemRing];
  int item[kItemRing];
  int4 tile[kItemRing];
};
__device__ __forceinline__ void tring_init(TileRing* r, int consumers) {
  for (int i = 0; i < kItemRing; ++i) {
    mbar_init(&r->full[i], 1);
    mbar_init(&r->empty[i], consumers);
  }
}
// A work tile {doc_start, len, prefix, first row} must lie inside the T packed tokens.
__device__ __forceinline__ bool tile_in_bounds(const int4& t, int T) {
  return t.x >= 0 && t.y > 0 && t.x + t.y <= T && t.w >= 0 && t.w < t.y && t.z >= 0 && t.z <= t.y;
}
__device__ __forceinline__ bool tring_push(TileRing* r, int k, int* counter, const int4* tiles, int H, int n_items,
                                           int T, int* err, int& item, int4& tile) {
  const int s = k % kItemRing;
  if (!mbar_wait(&r->empty[s], ((k / kItemRing) & 1) ^ 1)) return false;
  item = atomicAdd(counter, 1);
  tile = item < n_items ? tiles[item / H] : make_int4(0, 0, 0, 0);
  if (item < n_items && !HRM_BOUNDS_OK(tile_in_bounds(tile, T), err, 100)) item = n_items;  // every role stops
  *reinterpret_cast<volatile int*>(&r->item[s]) = item;
  r->tile[s] = tile;  // published by the release arrive below (the asm clobbers memory)
  mbar_arrive(&r->full[s]);
  return true;
}
__device__ __forceinline__ int tring_pop_thread(TileRing* r, int k, int4& tile) {
  const int s = k % kItemRing;
  if (!mbar_wait(&r->full[s], (k / kItemRing) & 1)) return INT_MAX;
  const int it = *reinterpret_cast<volatile int*>(&r->item[s]);
  tile = r->tile[s];
  mbar_arrive(&r->empty[s]);
  return it;
}
__device__ __forceinline__ int tring_pop_warp(TileRing* r, int k, int4& tile) {
  const int s = k % kItemRing;
  if (!__all_sync(0xffffffffu, mbar_wait(&r->full[s], (k / kItemRing) & 1))) return INT_MAX;
  const int it = *reinterpret_cast<volatile int*>(&r->item[s]);
  tile = r->tile[s];
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&r->empty[s]);
  return it;
}

struct Barriers {
  uint64_t q_full[2], q_empty[2];
  uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
  uint64_t s_full[2];
  uint64_t p_full[2], o_done[2], o_free, ml_full, drain;
  TileRing ring;
};

__global__ void __launch_bounds__(THREADS, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                       // 2 stages
  uint8_t* sK = smem + 2 * TILE_BYTES;      // 2 stages
  uint8_t* sV = smem + 4 * TILE_BYTES;      // 2 stages
  float2* sML = reinterpret_cast<float2*>(smem + 6 * TILE_BYTES);
  Barriers* bar = reinterpret_cast<Barriers*>(smem + 6 * TILE_BYTES + ML_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = p.sched[0];
  const int n_items = n_tiles * p.H;
  const int4* tiles = reinterpret_cast<const int4*>(p.sched + SCHED_HEADER);

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar->q_full[s], 1);
      mbar_init(&bar->q_empty[s], 1);
      mbar_init(&bar->k_full[s], 1);
      mbar_init(&bar->k_empty[s], 1);
      mbar_init(&bar->v_full[s], 1);
      mbar_init(&bar->v_empty[s], 1);
      mbar_init(&bar->s_full[s], 1);
      mbar_init(&bar->p_full[s], 128);
      mbar_init(&bar->o_done[s], 1);
    }
    mbar_init(&bar->o_free, 256);
    mbar_init(&bar->ml_full, 256);
    mbar_init(&bar->drain, 1);
    tring_init(&bar->ring, 9);  // UMMA thread + 8 softmax warps
    fence_mbar_init();
    tma_prefetch_desc(&tm_qkv);
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(tmem_slot, TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // number of 128-key blocks of a tile
  auto tile_blocks = [&](const int4& t) {
    const int kmax = min(t.y, max(t.z, t.w + BQ));
    return (kmax + BKV - 1) / BKV;
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA loads
    if (lane == 0) {
      int n = 0, kv = 0;
      int last_q[2] = {-1, -1}, last_k[2] = {-1, -1}, last_v[2] = {-1, -1};
      bool ok = true;
      for (int kk = 0; ok; ++kk, ++n) {
        int item;
        int4 t;
        if (!tring_push(&bar->ring, kk, const_cast<int*>(p.sched) + 4, tiles, p.H, n_items, p.T, p.err, item, t)) { report_error(p.err, kErrAttnWaitTimeout, 10); ok = false; break; }
        if (item >= n_items) break;
        const int head = item % p.H;
        const int qx = (p.H + head) * D, kx = (2 * p.H + head) * D, vx = (3 * p.H + head) * D;
        const int qs = n & 1;
        if (!mbar_wait(&bar->q_empty[qs], ((n >> 1) & 1) ^ 1)) { report_error(p.err, kErrAttnWaitTimeout, 11); ok = false; break; }
        mbar_arrive_expect_tx(&bar->q_full[qs], TILE_BYTES);
        tma_load_2d(sQ + qs * TILE_BYTES, &tm_qkv, &bar->q_full[qs], qx, t.x + t.w);
        tma_load_2d(sQ + qs * TILE_BYTES + TILE_BYTES / 2, &tm_qkv, &bar->q_full[qs], qx + 64, t.x + t.w);
        last_q[qs] = n >> 1;
        const int nb = tile_blocks(t);
        for (int j = 0; j < nb; ++j, ++kv) {
          const int s = kv & 1, r = kv >> 1;
          const int row = t.x + j * BKV;
          if (!mbar_wait(&bar->k_empty[s], (r & 1) ^ 1)) { report_error(p.err, kErrAttnWaitTimeout, 12); ok = false; break; }
          mbar_arrive_expect_tx(&bar->k_full[s], TILE_BYTES);
          tma_load_2d(sK + s * TILE_BYTES, &tm_qkv, &bar->k_full[s], kx, row);
          tma_load_2d(sK + s * TILE_BYTES + TILE_BYTES / 2, &tm_qkv, &bar->k_full[s], kx + 64, row);
          last_k[s] = r;
          if (!mbar_wait(&bar->v_empty[s], (r & 1) ^ 1)) { report_error(p.err, kErrAttnWaitTimeout, 13); ok = false; break; }
          mbar_arrive_expect_tx(&bar->v_full[s], TILE_BYTES);
          tma_load_2d(sV + s * TILE_BYTES, &tm_qkv, &bar->v_full[s], vx, row);
          tma_load_2d(sV + s * TILE_BYTES + TILE_BYTES / 2, &tm_qkv, &bar->v_full[s], vx + 64, row);
          last_v[s] = r;
        }
      }
      if (!ok) {  // drain this thread's copies in flight
        for (int s = 0; s < 2; ++s) {
          if (last_q[s] >= 0) mbar_wait(&bar->q_full[s], last_q[s] & 1);
          if (last_k[s] >= 0) mbar_wait(&bar->k_full[s], last_k[s] & 1);
          if (last_v[s] >= 0) mbar_wait(&bar->v_full[s], last_v[s] & 1);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- UMMA issue
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, 128, 0, 0);   // Q K^T: both K-major over d
      constexpr uint32_t idesc_pv = umma_idesc_bf16(128, 128, 0, 1);  // P V: P K-major over keys, V MN-major
      const uint32_t q_base = smem_u32(sQ), k_base = smem_u32(sK), v_base = smem_u32(sV);
      int n = 0, kv = 0;
      bool ok = true;
      auto wait_or_fail = [&](uint64_t* b, uint32_t par, int site) {
        if (mbar_wait(b, par)) return true;
        report_error(p.err, kErrAttnWaitTimeout, site);
        ok = false;
        return false;
      };
      // O_a += P[:, 0:64] V[0:64] and O_b += P[:, 64:128] V[64:128] for block `blk` (global
      // block counter) of stage s, each as soon as its softmax half has written P into TMEM
      // (half g: bf16 pairs in columns [g*64, g*64 + 32) of the block's S buffer, 8 columns
      // per 16 keys); the first block of an item overwrites both accumulators
      auto issue_pv = [&](int blk, bool first) -> bool {
        const int s = blk & 1, r = blk >> 1;
        if (!wait_or_fail(&bar->v_full[s], r & 1, 22)) return false;
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          if (!wait_or_fail(&bar->p_full[g], blk & 1, 21)) return false;
          tc_fence_after();
          const uint32_t p_tmem = tmem + (s ? TM_S1 : TM_S0) + g * 64;
#pragma unroll
          for (int k = 0; k < 4; ++k) {  // 16 keys per step
            const uint64_t b = umma_desc_sw128(v_base + s * TILE_BYTES + (g * 4 + k) * 2048, TILE_BYTES / 2, 1024);
            umma_f16_ts(tmem + (g ? TM_OB : TM_OA), p_tmem + k * 8, b, idesc_pv, (first && k == 0) ? 0u : 1u);
          }
          if (g == 1) umma_commit(&bar->v_empty[s]);
          umma_commit(&bar->o_done[g]);
        }
        return true;
      };
      for (int kk = 0; ok; ++kk, ++n) {
        int4 t;
        const int item = tring_pop_thread(&bar->ring, kk, t);
        if (item == INT_MAX) { report_error(p.err, kErrAttnWaitTimeout, 9); ok = false; break; }
        if (item >= n_items) break;
        const int nb = tile_blocks(t);
        const int qs = n & 1;
        if (!wait_or_fail(&bar->q_full[qs], (n >> 1) & 1, 23)) break;
        const uint32_t q_tile = q_base + qs * TILE_BYTES;
        const int first_blk = kv;
        for (int j = 0; j < nb && ok; ++j, ++kv) {
          const int s = kv & 1, r = kv >> 1;
          if (!wait_or_fail(&bar->k_full[s], r & 1, 24)) break;
          // buffer s held S/P of block kv-2, whose PV was issued above in program order
          tc_fence_after();
          const uint32_t d_s = tmem + (s ? TM_S1 : TM_S0);
#pragma unroll
          for (int k = 0; k < 8; ++k) {  // 16 dims per step
            const uint32_t off = (k >> 2) * (TILE_BYTES / 2) + (k & 3) * 32;
            umma_f16_ss(d_s, umma_desc_sw128(q_tile + off, 16, 1024),
                        umma_desc_sw128(k_base + s * TILE_BYTES + off, 16, 1024), idesc_s, k > 0 ? 1u : 0u);
          }
          umma_commit(&bar->k_empty[s]);
          umma_commit(&bar->s_full[s]);
          if (j == nb - 1) umma_commit(&bar->q_empty[qs]);
          if (j > 0) {
            if (j == 1 && !wait_or_fail(&bar->o_free, (n & 1) ^ 1, 26)) break;
            if (!issue_pv(kv - 1, j == 1)) break;
          }
        }
        if (!ok) break;
        if (nb == 1 && !wait_or_fail(&bar->o_free, (n & 1) ^ 1, 26)) break;
        if (!issue_pv(kv - 1, nb == 1)) break;
        (void)first_blk;
      }
      umma_commit(&bar->drain);
      mbar_wait(&bar->drain, 0);
    }
  } else {
    // ---------------------------------------------------------------- softmax / epilogue
    const int wg = (warp - 2) >> 2;  // key half of every block handled by this warpgroup
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tm_o = tmem + lane_off + (wg ? TM_OB : TM_OA);
    const float sl = p.scale_log2;
    int n = 0, kv = 0;
    bool ok = true;
    for (int kk = 0; ok; ++kk, ++n) {
      int4 t;
      const int item = tring_pop_warp(&bar->ring, kk, t);
      if (item == INT_MAX) { report_error(p.err, kErrAttnWaitTimeout, 8); ok = false; break; }
      if (item >= n_items) break;
      const int head = item % p.H;
      const int doc_start = t.x, len = t.y, prefix = t.z, q0 = t.w;
      const int nb = tile_blocks(t);
      const int qi = q0 + row;                         // doc-relative query of this thread
      const int limit = min(len, max(prefix, qi + 1));  // keys [0, limit) are visible
      const int full_until = min(len, max(prefix, q0 + 1));
      const bool row_ok = qi < len;
      const long tok = (long)doc_start + qi;
      // this row's 64 gate values of this half, fetched now and used by the epilogue
      uint4 gate[8];
      {
        const uint4* grow = reinterpret_cast<const uint4*>(p.qkv + (row_ok ? tok : 0) * p.ld_qkv + head * D + wg * 64);
#pragma unroll
        for (int q = 0; q < 8; ++q) gate[q] = row_ok ? __ldg(grow + q) : make_uint4(0, 0, 0, 0);
      }
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < nb; ++j, ++kv) {
        const int s = kv & 1;
        if (!warp_wait(&bar->s_full[s], (kv >> 1) & 1)) { report_error(p.err, kErrAttnWaitTimeout, 31); ok = false; break; }
        tc_fence_after();
        float v[64];
        {
          uint32_t r0[32], r1[32];
          const uint32_t ts = tmem + lane_off + (s ? TM_S1 : TM_S0) + wg * 64;
          tmem_ld_32x32b_x32(ts, r0);
          tmem_ld_32x32b_x32(ts + 32, r1);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            v[e] = __uint_as_float(r0[e]);
            v[e + 32] = __uint_as_float(r1[e]);
          }
        }
        const int kbase = j * BKV + wg * 64;
        if (kbase + 64 > full_until) {  // partially visible half-block (uniform per warpgroup)
#pragma unroll
          for (int e = 0; e < 64; ++e)
            if (kbase + e >= limit) v[e] = -INFINITY;
        }
        float mx0 = v[0], mx1 = v[1];
#pragma unroll
        for (int e = 2; e < 64; e += 2) {
          mx0 = fmaxf(mx0, v[e]);
          mx1 = fmaxf(mx1, v[e + 1]);
        }
        const float bmax = fmaxf(mx0, mx1) * sl;  // scale > 0 commutes with max
        // The rescale decision is per row, but tcgen05.ld/st are warp-collective
        // (.sync.aligned): decide per warp, and let rows that need no rescale use alpha = 1.
        const bool need = bmax > m_used + kRescaleThreshold;
        const bool rescale = __any_sync(0xffffffffu, need);
        float alpha = 1.f;
        if (rescale) {
          alpha = need ? fast_exp2(m_used - bmax) : 1.f;  // 0 on the first block
          if (need) {
            l *= alpha;
            m_used = bmax;
          }
        }
        // P = exp2(s * scale - m_used) as bf16 pairs, written over this half's S columns
        const float neg_m = m_used == -INFINITY ? 0.f : -m_used;
        float l0 = 0.f, l1 = 0.f;
        {
          uint32_t pk[32];
#pragma unroll
          for (int w = 0; w < 32; ++w) {
            const float p0 = fast_exp2(fmaf(v[2 * w], sl, neg_m));
            const float p1 = fast_exp2(fmaf(v[2 * w + 1], sl, neg_m));
            l0 += p0;
            l1 += p1;
            pk[w] = pack_bf16x2(p0, p1);
          }
          tmem_st_32x32b_x32(tmem + lane_off + (s ? TM_S1 : TM_S0) + wg * 64, pk);
        }
        l += l0 + l1;
        // O of this half may be rescaled only once PV_{kv-1} has landed; waiting every block
        // (PV_{kv-1} is long done in the steady state) keeps the barrier's phase in step
        if (!warp_wait(&bar->o_done[wg], (kv - 1) & 1)) { report_error(p.err, kErrAttnWaitTimeout, 32); ok = false; break; }
        tc_fence_after();
        if (rescale && j > 0) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tm_o + c * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
            tmem_st_32x32b_x32(tm_o + c * 32, r);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&bar->p_full[wg]);
      }
      if (!ok) break;
      // epilogue: wait for the last PV of both halves (O_b's commit follows O_a's), merge the
      // two partial softmax results, normalise, gate, write this half's 64 columns of O / Y
      if (!warp_wait(&bar->o_done[1], (kv - 1) & 1)) { report_error(p.err, kErrAttnWaitTimeout, 33); ok = false; break; }
      tc_fence_after();
      sML[wg * 128 + row] = make_float2(m_used, l);
      mbar_arrive(&bar->ml_full);
      if (!warp_wait(&bar->ml_full, n & 1)) { report_error(p.err, kErrAttnWaitTimeout, 34); ok = false; break; }
      const float2 oth = sML[(wg ^ 1) * 128 + row];
      const float m_all = fmaxf(m_used, oth.x);
      const float m_ref = m_all == -INFINITY ? 0.f : m_all;
      const float sc_me = fast_exp2(m_used - m_ref), sc_oth = fast_exp2(oth.x - m_ref);  // exp2(-inf) = 0
      const float l_all = l * sc_me + oth.y * sc_oth;
      const float inv = l_all > 0.f ? 1.f / l_all : 0.f;
      const float sa = (wg == 0 ? sc_me : sc_oth) * inv, sb = (wg == 0 ? sc_oth : sc_me) * inv;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int col = wg * 64 + c * 32;
        float va[32], vb[32];
        {
          uint32_t ra[32], rb[32];
          tmem_ld_32x32b_x32(tmem + lane_off + TM_OA + col, ra);
          tmem_ld_32x32b_x32(tmem + lane_off + TM_OB + col, rb);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            va[e] = __uint_as_float(ra[e]);
            vb[e] = __uint_as_float(rb[e]);
          }
        }
        if (row_ok) {
          __nv_bfloat16* orow = p.out + tok * p.ld_out + head * D + col;
          __nv_bfloat16* yrow = p.y + tok * p.ld_out + head * D + col;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 gv = gate[c * 4 + q];
            const uint32_t ga[4] = {gv.x, gv.y, gv.z, gv.w};
            uint32_t ow[4], yw[4];
#pragma unroll
            for (int w = 0; w < 4; ++w) {
              const int e = 8 * q + 2 * w;
              const float o0 = bf16_round(va[e] * sa + vb[e] * sb);
              const float o1 = bf16_round(va[e + 1] * sa + vb[e + 1] * sb);
              const float2 g = unpack_bf16x2(ga[w]);
              ow[w] = pack_bf16x2(o0, o1);
              yw[w] = pack_bf16x2(o0 * sigmoidf_(g.x), o1 * sigmoidf_(g.y));
            }
            reinterpret_cast<uint4*>(orow)[q] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
            reinterpret_cast<uint4*>(yrow)[q] = make_uint4(yw[0], yw[1], yw[2], yw[3]);
          }
        }
      }
      if (wg == 0 && row_ok) p.lse[(long)head * p.T + tok] = m_all + __log2f(l_all);
      tc_fence_before();
      mbar_arrive(&bar->o_free);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TM_COLS);
  }
  if (threadIdx.x == 0) finish_items(const_cast<int*>(p.sched) + 4, const_cast<int*>(p.sched) + 5);
}

// Zero O, Y and LSE of padding tokens [total, T).
__global__ void zero_tail_kernel(__nv_bfloat16* out, __nv_bfloat16* y, long ld_out, float* lse, int T, int H,
                                 const int* sched) {
  const int total = sched[2];
  const int chunks = H * D / 8;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < (long)(T - total) * chunks;
       i += (long)gridDim.x * blockDim.x) {
    const long tok = total + i / chunks;
    const int c = (int)(i % chunks) * 8;
    *reinterpret_cast<uint4*>(out + tok * ld_out + c) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(y + tok * ld_out + c) = make_uint4(0, 0, 0, 0);
  }
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < (long)(T - total) * H;
       i += (long)gridDim.x * blockDim.x)
    lse[(long)(i % H) * T + total + i / H] = 0.f;
}


// =======================================================================================
// Backward (tcgen05). One CTA = one 128-key block of one head at a time (pulled from the
// LPT-sorted key-block list), looping over the 64-query blocks that can see those keys. Per query block b:
//   S^T  = K Q^T      (M=128 keys, N=64 queries, K=128 dims)  -> TMEM region b % 2
//   dP^T = V dO^T     (same shape)                              -> TMEM region b % 2
//   softmax warps (row = key): P^T = exp2(S^T * scale_log2 - lse[q]) (masked to 0),
//     dS^T = P^T * (dP^T - D[q]) * scale  -> bf16, K-major swizzled smem tiles
//   dV  += P^T dO     (M=128 keys, N=128 dims, K=64 queries)   -> TMEM, whole key block
//   dK  += dS^T Q     (same shape)                              -> TMEM, whole key block
//   dQ^T = K^T dS^T   (M=128 dims, N=64 queries, K=128 keys)   -> TMEM, in the S^T columns
//     of region b % 2 (S^T of block b is already in the softmax warps' registers)
// The UMMA warp issues S^T / dP^T of block b+1 before the dV / dK / dQ^T products of block b,
// so the softmax of b+1 overlaps the tensor-core work of b (two TMEM regions).
// Warp roles (320 threads): 0 TMA, 1 UMMA, 2..9 compute. Compute warp group g (warps 2-5,
// 6-9) owns queries [32g, 32g+32) of every block: the softmax of that half (two warps per
// scheduler), then, before writing that block's P^T / dS^T, the previous block's dQ^T, which it
// moves from TMEM through a warp-private shared-memory box into the fp32 dQ accumulator with
// one tensor reduction per warp and block (cp.reduce.async.bulk.tensor .add, [32 x 32] fp32).
// P^T / dS^T tiles are double-buffered by block parity, so a block's softmax only waits for
// the UMMAs of the block two back; the dQ boxes of a block are staged in that block's consumed
// P^T / dS^T pair. At the end of the key block group 0 applies the RoPE backward to dK and
// writes it, group 1 writes dV.
// TMEM: S^T_0 [0,64), dP^T_0 [64,128), S^T_1 [128,192), dP^T_1 [192,256), dV [256,384),
// dK [384,512).
// Shared: K 32 KB, V 32 KB, Q 3x16 KB, dO 3x16 KB, 2 x (P^T 16 KB | dS^T 16 KB), lse/D 2 KB.
// =======================================================================================
constexpr int BWD_THREADS = 320;
constexpr int BQB = 64;                 // queries per block
constexpr int QTILE_BYTES = BQB * 128 * 2;   // [64][128] bf16 = two [64][64] boxes (16 KB)
constexpr int PTILE_BYTES = 128 * BQB * 2;   // [128 keys][64 queries] bf16 (16 KB)
constexpr int QSTAGES = 3;                   // Q / dO ring depth
// P^T | dS^T pairs are double-buffered by block parity, so the softmax of block b waits only for
// the UMMAs of block b - 2. A drained block's dQ^T is staged (per compute warp [32 queries][32
// dims] fp32) in that block's own, consumed, P^T | dS^T pair.
constexpr int PD_BYTES = 2 * PTILE_BYTES;
constexpr int DQ_STAGE_BYTES = 32 * 32 * 4;
static_assert(8 * DQ_STAGE_BYTES == PD_BYTES, "dQ staging aliases one P^T | dS^T pair");
// No alignment slack: with no static shared memory the dynamic window starts 1024-byte aligned
// (the kernel checks, and reports an error instead of running misaligned).
constexpr int BWD_SMEM_BYTES = 2 * TILE_BYTES + 2 * QSTAGES * QTILE_BYTES + 2 * PD_BYTES + 2048 + 512;
static_assert(BWD_SMEM_BYTES <= 232448, "backward exceeds the shared-memory limit");
constexpr uint32_t TB_S = 0, TB_DP = 64, TB_REGION = 128, TB_DV = 256, TB_DK = 384;

struct BwdParams {
  __nv_bfloat16* dqkv;
  long ld_dqkv;
  const float* lse;   // [H, T] log2 domain
  const float* dsum;  // [H, T]
  float* dq_acc;      // [T, H*128]
  const int* positions;
  const float* cos_tab;  // [S, 64]
  const float* sin_tab;
  int T, H;
  float scale, scale_log2;
  const int* sched;
  int cap;
  int* err;
  int profile;  // nonzero: accumulate per-phase clock counts into g_bwd_phase
  int rope_rows;  // rows of the cos / sin tables
};

// Phase tracing of the backward (off unless enabled from the host): cycles each role spends
// in each wait / work phase, summed over CTAs, read by attn_bwd_phase_counters().
constexpr int kBwdPhases = 20;
__device__ unsigned long long g_bwd_phase[kBwdPhases];
__device__ __forceinline__ unsigned long long cycle_clock() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(t));
  return t;
}
struct PhaseClock {
  bool on;
  unsigned long long t, acc[kBwdPhases];
  __device__ explicit PhaseClock(bool enabled) : on(enabled), t(enabled ? cycle_clock() : 0ull) {
#pragma unroll
    for (int i = 0; i < kBwdPhases; ++i) acc[i] = 0ull;
  }
  __device__ __forceinline__ void mark(int slot) {
    if (on) {
      const unsigned long long now = cycle_clock();
      acc[slot] += now - t;
      t = now;
    }
  }
  __device__ __forceinline__ void flush(int lo, int hi) {
    if (on)
      for (int i = lo; i < hi; ++i) atomicAdd(&g_bwd_phase[i], acc[i]);
  }
};

struct BwdBarriers {
  uint64_t kv_full, kv_done, kv_free;
  uint64_t qd_full[QSTAGES], qd_empty[QSTAGES];
  uint64_t s_full[2], dq_full[2], dq_free[2];
  uint64_t p_full[2], p_free[2], stage_free[2], drain;
  ItemRing ring;
};
static_assert(sizeof(BwdBarriers) + sizeof(uint32_t) <= 512, "backward barriers exceed their shared-memory slot");

// smem box -> global, element-wise fp32 add, through a tensor map (one instruction per box)
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(smem_u32(smem_src))
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_group_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ int bwd_qstart(const int4& t) { return t.w < t.z ? 0 : t.w; }
__device__ __forceinline__ int bwd_nqb(const int4& t) { return (t.y - bwd_qstart(t) + BQB - 1) / BQB; }

__global__ void __launch_bounds__(BWD_THREADS, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_kv, const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_do, const __grid_constant__ CUtensorMap tm_dq,
                       const BwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if ((smem_u32(smem_raw) & 1023u) != 0u) {  // the swizzled tiles need 1024-byte alignment
    if (threadIdx.x == 0) report_error(p.err, kErrAttnWaitTimeout, 65);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* sK = smem;
  uint8_t* sV = sK + TILE_BYTES;
  uint8_t* sQ = sV + TILE_BYTES;               // QSTAGES stages
  uint8_t* sDO = sQ + QSTAGES * QTILE_BYTES;   // QSTAGES stages
  uint8_t* sPD = sDO + QSTAGES * QTILE_BYTES;  // 2 x (P^T [16 KB] | dS^T [16 KB]), block parity
  float* sLse = reinterpret_cast<float*>(sPD + 2 * PD_BYTES);  // per compute warp: [32] lse, [32] D
  BwdBarriers* bar = reinterpret_cast<BwdBarriers*>(sLse + 512);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = p.sched[1] * p.H;
  const int4* tiles = reinterpret_cast<const int4*>(p.sched + SCHED_HEADER) + p.cap;

  if (threadIdx.x == 0) {
    mbar_init(&bar->kv_full, 1);
    mbar_init(&bar->kv_done, 1);
    mbar_init(&bar->kv_free, 256);
    for (int s = 0; s < QSTAGES; ++s) {
      mbar_init(&bar->qd_full[s], 1);
      mbar_init(&bar->qd_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar->s_full[s], 1);
      mbar_init(&bar->dq_full[s], 1);
      mbar_init(&bar->dq_free[s], 256);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar->p_full[s], 256);
      mbar_init(&bar->p_free[s], 1);
      mbar_init(&bar->stage_free[s], 8);  // lane 0 of each compute warp
    }
    mbar_init(&bar->drain, 1);
    ring_init(&bar->ring, 9);  // UMMA thread + 8 compute warps
    fence_mbar_init();
    tma_prefetch_desc(&tm_kv);
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_dq);
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(tmem_slot, TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA loads
    if (lane == 0) {
      int n = 0, qb_all = 0;
      int last_kv = -1, last_q[QSTAGES];
#pragma unroll
      for (int s = 0; s < QSTAGES; ++s) last_q[s] = -1;
      bool ok = true;
      for (int kk = 0; ok; ++kk, ++n) {
        int item;
        if (!ring_push(&bar->ring, kk, const_cast<int*>(p.sched) + 6, item)) { report_error(p.err, kErrAttnWaitTimeout, 40); ok = false; break; }
        if (item >= n_items) break;
        const int4 t = tiles[item / p.H];
        if (!HRM_BOUNDS_OK(tile_in_bounds(t, p.T), p.err, 101)) { ok = false; break; }
        const int head = item % p.H;
        const int qx = (p.H + head) * D, kx = (2 * p.H + head) * D, vx = (3 * p.H + head) * D;
        // K / V of this item can only land once the previous item's UMMAs are done with the
        // single K / V buffer; its first QSTAGES query blocks can be loaded before that (their
        // stages are freed by the previous item's blocks), so they are not held back by it.
        bool kv_issued = false;
        auto issue_kv = [&]() -> bool {
          if (!mbar_wait(&bar->kv_done, (n & 1) ^ 1)) { report_error(p.err, kErrAttnWaitTimeout, 41); return false; }
          mbar_arrive_expect_tx(&bar->kv_full, 2 * TILE_BYTES);
          const int krow = t.x + t.w;
          tma_load_2d(sK, &tm_kv, &bar->kv_full, kx, krow);
          tma_load_2d(sK + TILE_BYTES / 2, &tm_kv, &bar->kv_full, kx + 64, krow);
          tma_load_2d(sV, &tm_kv, &bar->kv_full, vx, krow);
          tma_load_2d(sV + TILE_BYTES / 2, &tm_kv, &bar->kv_full, vx + 64, krow);
          last_kv = n;
          kv_issued = true;
          return true;
        };
        const int qs = bwd_qstart(t), nqb = bwd_nqb(t);
        for (int qb = 0; qb < nqb; ++qb, ++qb_all) {
          // block qb's stage was last used by block qb - QSTAGES: of this item if qb >= QSTAGES,
          // which needs this item's K / V to have been issued
          if (!kv_issued && (qb >= QSTAGES || mbar_try_wait(&bar->kv_done, (n & 1) ^ 1))) {
            if (!issue_kv()) { ok = false; break; }
          }
          const int s = qb_all % QSTAGES, r = qb_all / QSTAGES;
          if (!mbar_wait(&bar->qd_empty[s], (r & 1) ^ 1)) { report_error(p.err, kErrAttnWaitTimeout, 42); ok = false; break; }
          mbar_arrive_expect_tx(&bar->qd_full[s], 2 * QTILE_BYTES);
          const int qrow = t.x + qs + qb * BQB;
          tma_load_2d(sQ + s * QTILE_BYTES, &tm_q, &bar->qd_full[s], qx, qrow);
          tma_load_2d(sQ + s * QTILE_BYTES + QTILE_BYTES / 2, &tm_q, &bar->qd_full[s], qx + 64, qrow);
          tma_load_2d(sDO + s * QTILE_BYTES, &tm_do, &bar->qd_full[s], head * D, qrow);
          tma_load_2d(sDO + s * QTILE_BYTES + QTILE_BYTES / 2, &tm_do, &bar->qd_full[s], head * D + 64, qrow);
          last_q[s] = r;
        }
        if (!ok) break;
        if (!kv_issued && !issue_kv()) { ok = false; break; }
      }
      if (!ok) {
        if (last_kv >= 0) mbar_wait(&bar->kv_full, last_kv & 1);
        for (int s = 0; s < QSTAGES; ++s)
          if (last_q[s] >= 0) mbar_wait(&bar->qd_full[s], last_q[s] & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- UMMA issue
    if (lane == 0) {
      constexpr uint32_t id_s = umma_idesc_bf16(128, 64, 0, 0);    // S^T, dP^T
      constexpr uint32_t id_kv = umma_idesc_bf16(128, 128, 0, 1);  // dV, dK
      constexpr uint32_t id_dq = umma_idesc_bf16(128, 64, 1, 1);   // dQ^T
      const uint32_t kb = smem_u32(sK), vb = smem_u32(sV), qb0 = smem_u32(sQ), db0 = smem_u32(sDO);
      const uint32_t pb = smem_u32(sPD), dsb = pb + PTILE_BYTES;
      int n = 0, b = 0;
      bool ok = true;
      PhaseClock pc(p.profile != 0);
      auto wait_ok = [&](uint64_t* x, uint32_t par, int site) {
        if (mbar_wait(x, par)) return true;
        report_error(p.err, kErrAttnWaitTimeout, site);
        ok = false;
        return false;
      };
      // dV, dK and dQ^T of block `bb` (global counter): Q / dO stage bb % QSTAGES, TMEM region bb % 2
      auto finish = [&](int bb, bool first) -> bool {
        const int s = bb & 1, qst = bb % QSTAGES;
        const uint32_t qs = qb0 + qst * QTILE_BYTES, ds = db0 + qst * QTILE_BYTES;
        const uint32_t pbb = pb + s * PD_BYTES, dsbb = dsb + s * PD_BYTES;  // block parity buffers
        pc.mark(13);
        if (!wait_ok(&bar->p_full[s], (bb >> 1) & 1, 54)) return false;
        pc.mark(11);
        if (first && !wait_ok(&bar->kv_free, (n & 1) ^ 1, 55)) return false;
        pc.mark(12);
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k) {  // 16 queries per step
          const uint64_t bo = umma_desc_sw128(ds + k * 2048, QTILE_BYTES / 2, 1024);
          const uint64_t bq = umma_desc_sw128(qs + k * 2048, QTILE_BYTES / 2, 1024);
          const uint32_t acc = (!first || k > 0) ? 1u : 0u;
          umma_f16_ss(tmem + TB_DV, umma_desc_sw128(pbb + k * 32, 16, 1024), bo, id_kv, acc);
          umma_f16_ss(tmem + TB_DK, umma_desc_sw128(dsbb + k * 32, 16, 1024), bq, id_kv, acc);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {  // 16 keys per step
          umma_f16_ss(tmem + s * TB_REGION + TB_S, umma_desc_sw128(kb + k * 2048, TILE_BYTES / 2, 1024),
                      umma_desc_sw128(dsbb + k * 2048, PTILE_BYTES, 1024), id_dq, k > 0);
        }
        umma_commit(&bar->qd_empty[qst]);
        umma_commit(&bar->p_free[s]);
        umma_commit(&bar->dq_full[s]);
        return true;
      };
      for (int kk = 0; ok; ++kk, ++n) {
        const int item = ring_pop_thread(&bar->ring, kk);
        if (item == INT_MAX) { report_error(p.err, kErrAttnWaitTimeout, 9); ok = false; break; }
        if (item >= n_items) break;
        const int4 t = tiles[item / p.H];
        if (!HRM_BOUNDS_OK(tile_in_bounds(t, p.T), p.err, 102)) { ok = false; break; }
        const int nqb = bwd_nqb(t);
        pc.mark(13);
        if (!wait_ok(&bar->kv_full, n & 1, 51)) break;
        pc.mark(14);
        for (int qb = 0; qb < nqb; ++qb, ++b) {
          const int s = b & 1, r = b >> 1, qst = b % QSTAGES;
          if (!wait_ok(&bar->qd_full[qst], (b / QSTAGES) & 1, 52)) break;
          pc.mark(8);
          // region s is free once dQ^T of block b - 2 has been read out of it (which implies
          // S^T / dP^T of b - 2 were consumed before it)
          if (!wait_ok(&bar->dq_free[s], (r & 1) ^ 1, 53)) break;
          pc.mark(9);
          tc_fence_after();
          const uint32_t qs = qb0 + qst * QTILE_BYTES, ds = db0 + qst * QTILE_BYTES;
          const uint32_t reg = tmem + s * TB_REGION;
#pragma unroll
          for (int k = 0; k < 8; ++k) {  // 16 dims per step
            const uint32_t oa = (k >> 2) * (TILE_BYTES / 2) + (k & 3) * 32;
            const uint32_t ob = (k >> 2) * (QTILE_BYTES / 2) + (k & 3) * 32;
            umma_f16_ss(reg + TB_S, umma_desc_sw128(kb + oa, 16, 1024), umma_desc_sw128(qs + ob, 16, 1024), id_s,
                        k > 0);
            umma_f16_ss(reg + TB_DP, umma_desc_sw128(vb + oa, 16, 1024), umma_desc_sw128(ds + ob, 16, 1024), id_s,
                        k > 0);
          }
          umma_commit(&bar->s_full[s]);
          pc.mark(10);
          if (qb > 0 && !finish(b - 1, qb == 1)) break;
        }
        if (!ok) break;
        if (!finish(b - 1, nqb == 1)) break;
        umma_commit(&bar->kv_done);
      }
      pc.mark(13);
      pc.flush(8, 15);
      umma_commit(&bar->drain);
      mbar_wait(&bar->drain, 0);
    }
  } else {
    // ------------------------------------------------ softmax, dQ and dK/dV epilogue (warps 2..9)
    // Warp group g = 0 / 1 handles queries [32g, 32g+32) of every 64-query block: its softmax
    // half (TMEM lanes = keys of this warp's quarter), then, once the UMMAs of that block are
    // done, its half of dQ^T (TMEM lanes = head dims of this warp's quarter). At the end of a
    // key block each group writes half of dK (RoPE backward) and half of dV.
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // key within the block (softmax), head dim (dQ)
    const uint32_t lo = (uint32_t)(quarter * 32) << 16;
    float* lse_b = sLse + (warp - 2) * 64;  // warp-private copy of this block's lse / D
    float* d_b = lse_b + 32;
    int n = 0, b = 0;
    bool ok = true;
    PhaseClock pc(p.profile != 0 && warp == 2);
    // dQ^T of block bb (TMEM region bb % 2), queries qbase + [32g, 32g+32) of item tile t
    auto drain_dq = [&](int bb, const int4& t, int head, int qbase) -> bool {
      const int sreg = bb & 1;
      pc.mark(7);
      if (!warp_wait(&bar->dq_full[sreg], (bb >> 1) & 1)) { report_error(p.err, kErrAttnWaitTimeout, 71); return false; }
      pc.mark(4);
      tc_fence_after();
      uint32_t r[32];
      tmem_ld_32x32b_x32(tmem + lo + sreg * TB_REGION + TB_S + g * 32, r);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&bar->dq_free[sreg]);  // TMEM region reusable: dQ^T is in registers
      // staging: this warp's 4 KB of block bb's P^T | dS^T pair, which its UMMAs (complete, see
      // dq_full) no longer read; no warp writes P^T(bb + 2) there before every warp's reduction
      // of this box has read it (stage_free[bb & 1])
      float* stage = reinterpret_cast<float*>(sPD + sreg * PD_BYTES) + (warp - 2) * (32 * 32);
#pragma unroll
      for (int e = 0; e < 32; ++e) stage[e * 32 + lane] = __uint_as_float(r[e]);
      fence_async_smem();
      __syncwarp();
      // one [32 queries][32 dims] fp32 box added into dQ; rows past the document receive the
      // exact zeros of their masked dS (rows past T are clipped by the tensor map)
      if (lane == 0) {
        tma_reduce_add_2d(&tm_dq, stage, head * D + quarter * 32, t.x + qbase + g * 32);
        bulk_commit_group();
      }
      pc.mark(5);
      return true;
    };
    for (int kk = 0; ok; ++kk, ++n) {
      const int item = ring_pop_warp(&bar->ring, kk);
      pc.mark(18);
      if (item == INT_MAX) { report_error(p.err, kErrAttnWaitTimeout, 8); ok = false; break; }
      if (item >= n_items) break;
      const int4 t = tiles[item / p.H];
      if (!HRM_BOUNDS_OK(tile_in_bounds(t, p.T), p.err, 103)) { ok = false; break; }
      const int head = item % p.H;
      const int doc_start = t.x, len = t.y, prefix = t.z, k0 = t.w;
      const int qs = bwd_qstart(t), nqb = bwd_nqb(t);
      const int key = k0 + row;
      const bool key_ok = key < len;
      int pos_k = key_ok ? p.positions[(long)doc_start + key] : 0;  // for the dK RoPE backward
      if (!HRM_BOUNDS_OK(pos_k >= 0 && pos_k < p.rope_rows, p.err, 105)) pos_k = 0;
      if (key_ok) {  // the rows are read at the end of the key block: have them in L2 by then
        asm volatile("prefetch.global.L2 [%0];" ::"l"(p.cos_tab + (long)pos_k * 64 + g * 32));
        asm volatile("prefetch.global.L2 [%0];" ::"l"(p.sin_tab + (long)pos_k * 64 + g * 32));
      }
      // lse / D of this lane's query of the first block; later blocks one block ahead
      float pre_l, pre_d;
      auto fetch = [&](int qbase) {
        const int q = qbase + g * 32 + lane;
        const bool qv = q < len;
        const long idx = (long)head * p.T + doc_start + q;
        pre_l = qv ? p.lse[idx] : 0.f;
        pre_d = qv ? p.dsum[idx] : 0.f;
      };
      fetch(qs);
      for (int qb = 0; qb < nqb; ++qb, ++b) {
        const int qbase = qs + qb * BQB;  // doc-relative first query of the block
        const int q0 = qbase + g * 32;    // first query of this warp's half
        __syncwarp();
        lse_b[lane] = pre_l;
        d_b[lane] = pre_d;
        __syncwarp();
        if (qb + 1 < nqb) fetch(qbase + BQB);  // consumed next iteration: latency overlaps this one
        const int sreg = b & 1;
        pc.mark(7);
        if (!warp_wait(&bar->s_full[sreg], (b >> 1) & 1)) { report_error(p.err, kErrAttnWaitTimeout, 61); ok = false; break; }
        pc.mark(0);
        if (pc.on) pc.acc[15] += 1;
        tc_fence_after();
        uint32_t rs[32], rd[32];
        const uint32_t reg = tmem + lo + sreg * TB_REGION + g * 32;
        tmem_ld_32x32b_x32(reg + TB_S, rs);
        tmem_ld_32x32b_x32(reg + TB_DP, rd);
        tmem_ld_wait();
        // every (key, query) pair of this half block visible: no per-element mask
        const bool full = (k0 + 128 <= len) && (q0 + 32 <= len) && (k0 + 128 <= max(prefix, q0 + 1));
        uint32_t pp[16], dd[16];
        if (full) {
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const float4 l4 = *reinterpret_cast<const float4*>(lse_b + e);
            const float4 d4 = *reinterpret_cast<const float4*>(d_b + e);
            const float p0 = fast_exp2(fmaf(__uint_as_float(rs[e]), p.scale_log2, -l4.x));
            const float p1 = fast_exp2(fmaf(__uint_as_float(rs[e + 1]), p.scale_log2, -l4.y));
            const float p2 = fast_exp2(fmaf(__uint_as_float(rs[e + 2]), p.scale_log2, -l4.z));
            const float p3 = fast_exp2(fmaf(__uint_as_float(rs[e + 3]), p.scale_log2, -l4.w));
            pp[e >> 1] = pack_bf16x2(p0, p1);
            pp[(e >> 1) + 1] = pack_bf16x2(p2, p3);
            dd[e >> 1] = pack_bf16x2(p0 * p.scale * (__uint_as_float(rd[e]) - d4.x),
                                     p1 * p.scale * (__uint_as_float(rd[e + 1]) - d4.y));
            dd[(e >> 1) + 1] = pack_bf16x2(p2 * p.scale * (__uint_as_float(rd[e + 2]) - d4.z),
                                           p3 * p.scale * (__uint_as_float(rd[e + 3]) - d4.w));
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            float pr[2], ds[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int j = e + u;
              const int q = q0 + j;
              const bool vis = key_ok && q < len && key < max(prefix, q + 1);
              pr[u] = vis ? fast_exp2(fmaf(__uint_as_float(rs[j]), p.scale_log2, -lse_b[j])) : 0.f;
              ds[u] = pr[u] * p.scale * (__uint_as_float(rd[j]) - d_b[j]);
            }
            pp[e >> 1] = pack_bf16x2(pr[0], pr[1]);
            dd[e >> 1] = pack_bf16x2(ds[0], ds[1]);
          }
        }
        pc.mark(1);
        // dQ^T of block b - 1 first (its UMMAs ran while this block's softmax did): that frees
        // the TMEM region the UMMAs of block b + 1 need; its staging is pair (b - 1) & 1, not
        // the pair P^T(b) goes to
        if (qb > 0 && !drain_dq(b - 1, t, head, qbase - BQB)) { ok = false; break; }
        // pair b & 1 was last read by the UMMAs of block b - 2 ...
        if (!warp_wait(&bar->p_free[b & 1], ((b >> 1) & 1) ^ 1)) { report_error(p.err, kErrAttnWaitTimeout, 62); ok = false; break; }
        // ... and staged dQ^T(b - 2) for every warp's reduction
        if (b >= 2) {
          if (lane == 0) {
            // this warp's reduction of dQ^T(b - 2) has read its box (dQ^T(b - 1), committed
            // after it, may still be reading)
            bulk_wait_group_read1();
            mbar_arrive(&bar->stage_free[b & 1]);
          }
          if (!warp_wait(&bar->stage_free[b & 1], ((b - 2) >> 1) & 1)) { report_error(p.err, kErrAttnWaitTimeout, 64); ok = false; break; }
        }
        pc.mark(2);
        uint8_t* prow = sPD + (b & 1) * PD_BYTES + row * 128;
        uint8_t* drow = prow + PTILE_BYTES;
#pragma unroll
        for (int i = 0; i < 4; ++i) {  // 16-byte pieces g*4 + i of the 128-byte swizzled row
          const int off = ((g * 4 + i) ^ (row & 7)) << 4;
          *reinterpret_cast<uint4*>(prow + off) = make_uint4(pp[4 * i], pp[4 * i + 1], pp[4 * i + 2], pp[4 * i + 3]);
          *reinterpret_cast<uint4*>(drow + off) = make_uint4(dd[4 * i], dd[4 * i + 1], dd[4 * i + 2], dd[4 * i + 3]);
        }
        fence_async_smem();
        tc_fence_before();
        mbar_arrive(&bar->p_full[b & 1]);
        pc.mark(3);
      }
      if (!ok) break;
      if (!drain_dq(b - 1, t, head, qs + (nqb - 1) * BQB)) { ok = false; break; }
      pc.mark(7);
      // dK (RoPE backward) and dV of this key block, split between the two groups
      if (!warp_wait(&bar->kv_done, n & 1)) { report_error(p.err, kErrAttnWaitTimeout, 63); ok = false; break; }
      pc.mark(16);
      tc_fence_after();
      const long tok = (long)doc_start + key;
      // group g: dK dims [32g, 32g+32) with their RoPE partners +64, and dV dims [64g, 64g+64);
      // 16 dims per step with vector loads of cos / sin keep the loads in flight together
      {
        __nv_bfloat16* dk_row = p.dqkv + tok * p.ld_dqkv + (2 * p.H + head) * D;
        __nv_bfloat16* dv_row = p.dqkv + tok * p.ld_dqkv + (3 * p.H + head) * D;
        const float4* c4 = reinterpret_cast<const float4*>(p.cos_tab + (long)pos_k * 64 + g * 32);
        const float4* s4 = reinterpret_cast<const float4*>(p.sin_tab + (long)pos_k * 64 + g * 32);
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          const int d0 = g * 32 + h * 16;
          uint32_t r1[16], r2[16];
          tmem_ld_32x32b_x16(tmem + lo + TB_DK + d0, r1);
          tmem_ld_32x32b_x16(tmem + lo + TB_DK + 64 + d0, r2);
          float cs[16], sn[16];
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const float4 a = key_ok ? c4[h * 4 + v] : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 b = key_ok ? s4[h * 4 + v] : make_float4(0.f, 0.f, 0.f, 0.f);
            cs[4 * v] = a.x; cs[4 * v + 1] = a.y; cs[4 * v + 2] = a.z; cs[4 * v + 3] = a.w;
            sn[4 * v] = b.x; sn[4 * v + 1] = b.y; sn[4 * v + 2] = b.z; sn[4 * v + 3] = b.w;
          }
          tmem_ld_wait();
          if (key_ok) {
            uint32_t a[8], bb[8];
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              const float x1a = __uint_as_float(r1[e]), x1b = __uint_as_float(r1[e + 1]);
              const float x2a = __uint_as_float(r2[e]), x2b = __uint_as_float(r2[e + 1]);
              a[e >> 1] = pack_bf16x2(x1a * cs[e] + x2a * sn[e], x1b * cs[e + 1] + x2b * sn[e + 1]);
              bb[e >> 1] = pack_bf16x2(x2a * cs[e] - x1a * sn[e], x2b * cs[e + 1] - x1b * sn[e + 1]);
            }
            uint4* o1 = reinterpret_cast<uint4*>(dk_row + d0);
            uint4* o2 = reinterpret_cast<uint4*>(dk_row + 64 + d0);
            o1[0] = make_uint4(a[0], a[1], a[2], a[3]);
            o1[1] = make_uint4(a[4], a[5], a[6], a[7]);
            o2[0] = make_uint4(bb[0], bb[1], bb[2], bb[3]);
            o2[1] = make_uint4(bb[4], bb[5], bb[6], bb[7]);
          }
        }
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          const int d0 = g * 64 + c * 32;
          uint32_t rv[32];
          tmem_ld_32x32b_x32(tmem + lo + TB_DV + d0, rv);
          tmem_ld_wait();
          if (key_ok) {
            uint32_t va[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) va[e >> 1] = pack_bf16x2(__uint_as_float(rv[e]), __uint_as_float(rv[e + 1]));
            uint4* o = reinterpret_cast<uint4*>(dv_row + d0);
#pragma unroll
            for (int q = 0; q < 4; ++q) o[q] = make_uint4(va[4 * q], va[4 * q + 1], va[4 * q + 2], va[4 * q + 3]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&bar->kv_free);
      pc.mark(17);
    }
    if (lane == 0) bulk_wait_group0();
    if (lane == 0) pc.flush(0, 8);
    if (lane == 0) pc.flush(16, 20);
    if (lane == 0 && pc.on) atomicAdd(&g_bwd_phase[15], pc.acc[15]);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TM_COLS);
  }
  if (threadIdx.x == 0) finish_items(const_cast<int*>(p.sched) + 6, const_cast<int*>(p.sched) + 7);
}

}  // namespace attn_tc

at::Tensor device_error_word();

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn_attn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    TORCH_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
                    ptr != nullptr,
                "cuTensorMapEncodeTiled is unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}
}  // namespace

void attn_fwd_tc(const at::Tensor& qkv, int64_t H, const at::Tensor& sched, const at::Tensor& out,
                 const at::Tensor& y, const at::Tensor& lse) {
  c10::cuda::CUDAGuard guard(qkv.device());
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.stride(1) == 1, "qkv must be row-major bf16");
  TORCH_CHECK((qkv.stride(0) * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(qkv.data_ptr()) & 15) == 0,
              "qkv rows must be 16-byte aligned");
  TORCH_CHECK(qkv.size(1) >= 4 * H * attn_tc::D, "qkv width");
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int T = (int)qkv.size(0);

  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)qkv.size(1), (cuuint64_t)T};
  cuuint64_t strides[1] = {(cuuint64_t)(qkv.stride(0) * 2)};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn_attn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, qkv.data_ptr(), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);

  attn_tc::Params p{};
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.y = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  p.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  TORCH_CHECK(out.stride(0) == y.stride(0), "O and Y must share a row stride");
  p.ld_out = out.stride(0);
  p.ld_qkv = qkv.stride(0);
  p.lse = lse.data_ptr<float>();
  p.T = T;
  p.H = (int)H;
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)attn_tc::D));
  p.sched = sched.data_ptr<int>();
  p.err = device_error_word().data_ptr<int>();

  TORCH_CHECK(ensure_dynamic_smem((const void*)attn_tc::attn_fwd_tc_kernel, attn_tc::SMEM_BYTES) == cudaSuccess,
              "cudaFuncSetAttribute failed");
  const int sms = device_sm_count();
  attn_tc::attn_fwd_tc_kernel<<<sms, attn_tc::THREADS, attn_tc::SMEM_BYTES, stream>>>(map, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  attn_tc::zero_tail_kernel<<<64, 256, 0, stream>>>(p.out, p.y, p.ld_out, p.lse, T, (int)H, p.sched);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}


namespace attn {
__global__ void attn_bwd_pre_kernel(const __nv_bfloat16* dy, const __nv_bfloat16* out, long ld_out,
                                    const __nv_bfloat16* qkv, long ld_qkv, __nv_bfloat16* d_out,
                                    __nv_bfloat16* dqkv, long ld_dqkv, float* dsum, float* dq_acc, int T, int H);
__global__ void attn_bwd_post_kernel(const float* dq_acc, __nv_bfloat16* dqkv, long ld_dqkv, const int* positions,
                                     const float* cos_tab, const float* sin_tab, int rope_rows, int* err, int T, int H,
                                     const int* sched);
}  // namespace attn

static CUtensorMap make_map_rows(const at::Tensor& t, uint32_t box_rows) {
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)t.size(1), (cuuint64_t)t.size(0)};
  cuuint64_t strides[1] = {(cuuint64_t)(t.stride(0) * 2)};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  TORCH_CHECK(t.scalar_type() == at::kBFloat16 && t.stride(1) == 1 && (t.stride(0) * 2) % 16 == 0 &&
                  (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0,
              "attention operands must be 16-byte aligned row-major bf16");
  CUresult r = encode_fn_attn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, t.data_ptr(), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return map;
}

static bool g_bwd_profile_enabled = false;

// Phase tracing of the tcgen05 attention backward: enable / disable, and read (optionally
// zeroing) the 16 per-phase cycle counters summed over CTAs (slot meanings in attention.py).
void attn_bwd_set_profile(bool enabled) { g_bwd_profile_enabled = enabled; }
at::Tensor attn_bwd_phase_counters(bool reset) {
  unsigned long long host[attn_tc::kBwdPhases];
  TORCH_CHECK(cudaMemcpyFromSymbol(host, attn_tc::g_bwd_phase, sizeof(host)) == cudaSuccess, "read phase counters");
  if (reset) {
    unsigned long long zero[attn_tc::kBwdPhases] = {};
    TORCH_CHECK(cudaMemcpyToSymbol(attn_tc::g_bwd_phase, zero, sizeof(zero)) == cudaSuccess, "reset phase counters");
  }
  auto out = at::empty({attn_tc::kBwdPhases}, at::TensorOptions().dtype(at::kLong));
  for (int i = 0; i < attn_tc::kBwdPhases; ++i) out[i] = (int64_t)host[i];
  return out;
}

void attn_bwd_tc(const at::Tensor& qkv, int64_t H, const at::Tensor& sched, const at::Tensor& out,
                 const at::Tensor& lse, const at::Tensor& dy, const at::Tensor& positions, const at::Tensor& cos_tab,
                 const at::Tensor& sin_tab, const at::Tensor& d_out, const at::Tensor& dsum, const at::Tensor& dq_acc,
                 const at::Tensor& dqkv) {
  c10::cuda::CUDAGuard guard(qkv.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int T = (int)qkv.size(0);
  auto bf = [](const at::Tensor& x) { return reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()); };
  auto bfm = [](const at::Tensor& x) { return reinterpret_cast<__nv_bfloat16*>(x.data_ptr()); };
  {
    const long warps = (long)T * H;
    const long blocks = (warps * 32 + 255) / 256;
    attn::attn_bwd_pre_kernel<<<(unsigned)blocks, 256, 0, stream>>>(
        bf(dy), bf(out), out.stride(0), bf(qkv), qkv.stride(0), bfm(d_out), bfm(dqkv), dqkv.stride(0),
        dsum.data_ptr<float>(), dq_acc.data_ptr<float>(), T, (int)H);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  const CUtensorMap m_kv = make_map_rows(qkv, 128), m_q = make_map_rows(qkv, 64), m_do = make_map_rows(d_out, 64);
  CUtensorMap m_dq;
  {
    TORCH_CHECK(dq_acc.scalar_type() == at::kFloat && dq_acc.is_contiguous() && dq_acc.size(1) == H * attn_tc::D &&
                    (reinterpret_cast<uintptr_t>(dq_acc.data_ptr()) & 15) == 0,
                "dq_acc must be a contiguous fp32 [T, H*128] buffer");
    cuuint64_t dims[2] = {(cuuint64_t)dq_acc.size(1), (cuuint64_t)dq_acc.size(0)};
    cuuint64_t strides[1] = {(cuuint64_t)(dq_acc.stride(0) * 4)};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn_attn()(&m_dq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, dq_acc.data_ptr(), dims, strides, box,
                                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (dQ) failed: ", (int)r);
  }
  attn_tc::BwdParams p{};
  p.dqkv = bfm(dqkv);
  p.ld_dqkv = dqkv.stride(0);
  p.lse = lse.data_ptr<float>();
  p.dsum = dsum.data_ptr<float>();
  p.dq_acc = dq_acc.data_ptr<float>();
  p.positions = positions.data_ptr<int>();
  p.cos_tab = cos_tab.data_ptr<float>();
  p.rope_rows = (int)cos_tab.size(0);
  p.sin_tab = sin_tab.data_ptr<float>();
  p.T = T;
  p.H = (int)H;
  p.scale = (float)(1.0 / std::sqrt(128.0));
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt(128.0));
  p.sched = sched.data_ptr<int>();
  p.cap = (int)((sched.numel() - attn_tc::SCHED_HEADER) / 8);
  p.err = device_error_word().data_ptr<int>();
  p.profile = g_bwd_profile_enabled ? 1 : 0;
  TORCH_CHECK(ensure_dynamic_smem((const void*)attn_tc::attn_bwd_tc_kernel, attn_tc::BWD_SMEM_BYTES) == cudaSuccess,
              "cudaFuncSetAttribute failed");
  const int sms = device_sm_count();
  attn_tc::attn_bwd_tc_kernel<<<sms, attn_tc::BWD_THREADS, attn_tc::BWD_SMEM_BYTES, stream>>>(m_kv, m_q, m_do, m_dq,
                                                                                               p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  attn::attn_bwd_post_kernel<<<1024, 256, 0, stream>>>(p.dq_acc, p.dqkv, p.ld_dqkv, p.positions, p.cos_tab, p.sin_tab,
                                                       (int)cos_tab.size(0), p.err, T, (int)H, p.sched);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace hrm

// ---------------------------------------------------------------------------------------
// Allocation-free attention forward (declared in attention_noalloc.h; no counterpart in the
// reference). It runs the same tcgen05 forward as attn_fwd_tc above; the work schedule and
// the error word live in the file-scope device array below instead of in memory that a
// caller or torch allocates.
// ---------------------------------------------------------------------------------------
#include "attention_noalloc.h"

namespace hrm {
namespace attn {
__global__ void schedule_kernel(const int* cu, const int* prefix_lens, int n_cu, int causal, int cap, int T,
                                int* sched, int* err);
}  // namespace attn
namespace attn_tc {
// Ints [0, kNoallocErrOffset): the schedule (header, forward and backward tile lists, 8 ints
// per tile); then the 4-int error word. One copy per GPU that loads the library.
static __device__ __align__(256) int g_noalloc_scratch[HRM_ATTN_NOALLOC_SCRATCH_BYTES / 4];
constexpr int kNoallocErrOffset = SCHED_HEADER + 8 * HRM_ATTN_NOALLOC_MAX_TILES;
static_assert(kNoallocErrOffset % 4 == 0 && kNoallocErrOffset + 4 <= HRM_ATTN_NOALLOC_SCRATCH_BYTES / 4,
              "allocation-free scratch layout");
}  // namespace attn_tc
}  // namespace hrm

namespace {
struct NoallocDevice {
  std::atomic<int*> scratch{nullptr};  // published last (release), after `sms`
  int sms = 0;
};
NoallocDevice g_noalloc[hrm::kMaxDevices];
std::mutex g_noalloc_mu;

// Once per device, with that device current: the static array's device address (host code
// must not use the symbol itself as a pointer), the kernel's shared-memory limit and the SM
// count. Host threads that race on the first call serialise on the mutex.
cudaError_t noalloc_setup(int dev, int** scratch, int* sms) {
  int* ptr = g_noalloc[dev].scratch.load(std::memory_order_acquire);
  if (ptr == nullptr) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    ptr = g_noalloc[dev].scratch.load(std::memory_order_relaxed);
    if (ptr == nullptr) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, hrm::attn_tc::g_noalloc_scratch);
      if (e != cudaSuccess) return e;
      e = hrm::ensure_dynamic_smem((const void*)hrm::attn_tc::attn_fwd_tc_kernel, hrm::attn_tc::SMEM_BYTES);
      if (e != cudaSuccess) return e;
      int n = 0;
      e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return e;
      g_noalloc[dev].sms = n;
      ptr = static_cast<int*>(p);
      g_noalloc[dev].scratch.store(ptr, std::memory_order_release);
    }
  }
  *scratch = ptr;
  *sms = g_noalloc[dev].sms;
  return cudaSuccess;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point, without exceptions.
CUresult noalloc_encode(CUtensorMap* map, void* base, int width, int T, long long ld) {
  using EncodeTiledFn = hrm::EncodeTiledFn;
  static std::atomic<EncodeTiledFn> fn{nullptr};
  EncodeTiledFn f = fn.load(std::memory_order_acquire);
  if (f == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        ptr == nullptr)
      return CUDA_ERROR_NOT_FOUND;
    f = reinterpret_cast<EncodeTiledFn>(ptr);
    fn.store(f, std::memory_order_release);
  }
  cuuint64_t dims[2] = {(cuuint64_t)width, (cuuint64_t)T};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  return f(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

template <typename... P, typename... A>
cudaError_t noalloc_launch(void (*kernel)(P...), int grid, int block, int smem, cudaStream_t stream, A&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<A>(args)...);
}
}  // namespace

extern "C" __attribute__((visibility("default"))) const char* hrm_attn_fwd_noalloc_strerror(int code) {
  if (code == 0) return "success";
  if (code == HRM_ATTN_NOALLOC_TOO_LARGE)
    return "problem too large for the static scratch: need ceil(T/128) + n_cu <= HRM_ATTN_NOALLOC_MAX_TILES";
  if (code == HRM_ATTN_NOALLOC_BAD_ARG)
    return "invalid argument (null or misaligned pointer, head count, row stride or device index)";
  if (code == HRM_ATTN_NOALLOC_TENSOR_MAP) return "cuTensorMapEncodeTiled rejected the qkv layout";
  return cudaGetErrorString(static_cast<cudaError_t>(code));
}

extern "C" __attribute__((visibility("default"))) int hrm_attn_fwd_noalloc(
    const void* qkv, long long ld_qkv, int T, int num_heads, const int* cu_seqlens, int n_cu, const int* prefix_lens,
    int causal, void* out, void* y, long long ld_out, float* lse, cudaStream_t stream) {
  const uintptr_t vec = reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(out) |
                        reinterpret_cast<uintptr_t>(y);
  const uintptr_t word = reinterpret_cast<uintptr_t>(lse) | reinterpret_cast<uintptr_t>(cu_seqlens) |
                         reinterpret_cast<uintptr_t>(prefix_lens);
  if (qkv == nullptr || cu_seqlens == nullptr || prefix_lens == nullptr || out == nullptr || y == nullptr ||
      lse == nullptr || T <= 0 || num_heads <= 0 || n_cu < 1 ||
      ld_qkv < 4LL * num_heads * hrm::attn_tc::D || ld_out < (long long)num_heads * hrm::attn_tc::D ||
      (ld_qkv % 8) != 0 || (ld_out % 8) != 0 || (vec & 15) != 0 || (word & 3) != 0)
    return HRM_ATTN_NOALLOC_BAD_ARG;
  const long long tiles = (T + 127) / 128 + (long long)n_cu;
  if (tiles > HRM_ATTN_NOALLOC_MAX_TILES) return HRM_ATTN_NOALLOC_TOO_LARGE;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= hrm::kMaxDevices) return HRM_ATTN_NOALLOC_BAD_ARG;
  int* scratch = nullptr;
  int sms = 0;
  e = noalloc_setup(dev, &scratch, &sms);
  if (e != cudaSuccess) return (int)e;

  CUtensorMap map;
  if (noalloc_encode(&map, const_cast<void*>(qkv), 4 * num_heads * hrm::attn_tc::D, T, ld_qkv) != CUDA_SUCCESS)
    return HRM_ATTN_NOALLOC_TENSOR_MAP;

  int* sched = scratch;
  int* err = scratch + hrm::attn_tc::kNoallocErrOffset;
  hrm::attn_tc::Params p{};
  p.out = static_cast<__nv_bfloat16*>(out);
  p.y = static_cast<__nv_bfloat16*>(y);
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
  p.ld_out = (long)ld_out;
  p.ld_qkv = (long)ld_qkv;
  p.lse = lse;
  p.T = T;
  p.H = num_heads;
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)hrm::attn_tc::D));
  p.sched = sched;
  p.err = err;

  // Each step returns its own launch status (no cudaGetLastError: that would also report,
  // and clear, an error left by some other caller on this thread).
  e = cudaMemsetAsync(err, 0, 4 * sizeof(int), stream);  // the error word starts at zero every call
  if (e != cudaSuccess) return (int)e;
  e = noalloc_launch(hrm::attn::schedule_kernel, 1, 1024, 0, stream, cu_seqlens, prefix_lens, n_cu,
                     causal ? 1 : 0, (int)HRM_ATTN_NOALLOC_MAX_TILES, T, sched, err);
  if (e != cudaSuccess) return (int)e;
  e = noalloc_launch(hrm::attn_tc::attn_fwd_tc_kernel, sms, hrm::attn_tc::THREADS, hrm::attn_tc::SMEM_BYTES, stream,
                     map, p);
  if (e != cudaSuccess) return (int)e;
  e = noalloc_launch(hrm::attn_tc::zero_tail_kernel, 64, 256, 0, stream, p.out, p.y, p.ld_out, p.lse, T, num_heads,
                     (const int*)sched);
  return (int)e;
}

extern "C" __attribute__((visibility("default"))) int hrm_attn_fwd_noalloc_status(int* code4) {
  if (code4 == nullptr) return HRM_ATTN_NOALLOC_BAD_ARG;
  const cudaError_t e = cudaMemcpyFromSymbol(code4, hrm::attn_tc::g_noalloc_scratch, 4 * sizeof(int),
                                             hrm::attn_tc::kNoallocErrOffset * sizeof(int), cudaMemcpyDeviceToHost);
  return (int)e;
}
