// Persistent warp-specialised bf16 GEMM on 5th-generation tensor cores (tcgen05, sm_100a).
//
//   D[M, N] = sum_k A(m, k) * B(n, k)       (fp32 accumulation in TMEM)
//
// Operands are row-major tensors; each may be "K-major" (reduction dim contiguous) or
// "MN-major" (output dim contiguous), which covers the three GEMMs of a linear layer:
//   forward  Y  = X  W^T : A = X [M,K]  K-major,  B = W [N,K]  K-major
//   dgrad    dX = dY W   : A = dY [M,N] K-major,  B = W [N,K]  MN-major (as [red, out])
//   wgrad    dW = dY^T X : A = dY [T,N] MN-major, B = X [T,K]  MN-major
//
// CTA tile 128 x 256 x 64, 4-stage TMA ring (48 KB / stage, 128B swizzle), one CTA per SM.
// Warp roles (320 threads):
//   warp 0      : TMA producer (one elected lane)
//   warp 1      : TMEM allocator + UMMA issuer (one elected lane)
//   warps 2..9  : epilogue; TMEM lane quarter = warp % 4, one accumulator row per thread;
//                 warps 2-5 and 6-9 split the tile's columns (two warps per lane quarter)
// The accumulator is double-buffered in TMEM (2 x 256 columns), so the epilogue of tile i
// overlaps the main loop of tile i+1.
//
// Work split: whole tiles strided over CTAs, or (fp32 atomic epilogue only) an even split of
// the flattened (tile, k-block) iteration space over CTAs ("stream-K"), which keeps every SM
// busy for the small-output / long-K weight-gradient GEMMs.
//
// Epilogues (fused; one pass over the accumulator):
//   STORE     out bf16 = acc
//   RESIDUAL  out bf16 = acc + residual
//   F32ADD    out fp32 += acc (atomic, stream-K)
//   ROPE      out bf16 = acc, with rotate-half RoPE on the q/k head columns
//   SWIGLU    B rows are gate/up pairs; writes gate|up and silu(gate)*up
//   SWIGLU_BWD acc = dh; reads gate|up, writes d(gate)|d(up)
//   CE        out bf16 logits + per-row partial (max, sum exp, argmax, target logit) per
//             128-column half tile
//
// All mbarrier waits are bounded (common.cuh); on a timeout the kernel records an error,
// drains its own TMA loads and UMMAs, frees TMEM and returns.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "collective_jobs.cuh"
#include "common.cuh"
#include "device_setup.h"

namespace hrm {

enum GemmEpilogue : int {
  EPI_STORE = 0,
  EPI_RESIDUAL = 1,
  EPI_F32ADD = 2,
  EPI_ROPE = 3,
  EPI_SWIGLU = 4,
  EPI_SWIGLU_BWD = 5,
  EPI_CE = 6,
  EPI_CE_BWD = 8,  // recomputed logits -> (softmax - onehot) * dloss, bf16 (one V chunk of the LM head)
};

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_STAGE_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_STAGE_BYTES = BN * BK * 2;  // 32 KB
constexpr int EPI_WARPS = 8;
constexpr int GEMM_THREADS = 64 + 32 * EPI_WARPS;
constexpr int TMEM_COLS = 2 * BN;
// bf16 outputs leave through TMA tensor stores: each epilogue warp stages a 32 x 32 box
// (64-byte rows, 64B-swizzled) in one of its two 2 KB buffers
// (only the epilogues with bf16 outputs reserve it: the fp32 weight-gradient GEMMs measured
// 30-45 % slower with the extra 32 KB of shared memory they do not use)
constexpr int STG_BOX_BYTES = 32 * 32 * 2;
constexpr int STG_BYTES = EPI_WARPS * 2 * STG_BOX_BYTES;  // 32 KB
template <int EPI>
constexpr bool stages_output() {
  return EPI == EPI_STORE || EPI == EPI_RESIDUAL || EPI == EPI_ROPE || EPI == EPI_SWIGLU || EPI == EPI_SWIGLU_BWD ||
         EPI == EPI_CE_BWD;
}
// The SwiGLU backward also brings its g / u inputs in through TMA: each warp holds two
// (g | u) box pairs (8 KB), and the main loop keeps fewer stages to make room (K is the hidden
// size, 20 k-blocks at L): 5 pair stages (231.9 KB) measured 0.194 ms at L against 0.201 ms
// with 4.
template <int EPI>
constexpr int stage_bytes() { return EPI == EPI_SWIGLU_BWD ? 2 * STG_BYTES : stages_output<EPI>() ? STG_BYTES : 0; }
template <int EPI>
constexpr int single_stages() { return EPI == EPI_SWIGLU_BWD ? 3 : STAGES; }
template <int EPI>
constexpr int pair_stages() { return EPI == EPI_SWIGLU_BWD ? 5 : 6; }
constexpr int BAR_BYTES = 512;  // mbarriers + TMEM slot
template <int EPI>
constexpr int gemm_smem_bytes() {
  return 1024 + single_stages<EPI>() * (A_STAGE_BYTES + B_STAGE_BYTES) + stage_bytes<EPI>() + BAR_BYTES;
}
static_assert(gemm_smem_bytes<0>() <= 232448 && gemm_smem_bytes<5>() <= 232448, "GEMM exceeds shared memory");
// CTA-pair (cta_group::2) variant: a 256 x 256 tile per pair of SMs, each SM stages its 128
// rows of A and its 128 columns of B, so a k-block costs each SM 32 KB instead of 48 KB of
// operand traffic for the same tensor-core work; 6 stages fit the same shared memory.
template <int EPI>
constexpr int pair_smem_bytes() {
  return 1024 + pair_stages<EPI>() * (A_STAGE_BYTES + B_STAGE_BYTES / 2) + stage_bytes<EPI>() + BAR_BYTES;
}
static_assert(pair_smem_bytes<0>() <= 232448 && pair_smem_bytes<5>() <= 232448, "pair GEMM exceeds shared memory");

struct GemmArgs {
  int M, N, K;
  void* out;
  long ldo;
  const __nv_bfloat16* residual;
  long ldr;
  void* out2;
  long ldo2;
  const __nv_bfloat16* aux;
  long ldaux;
  // RoPE (head_dim 128): fp32 tables [max_pos, 64]
  const int* positions;
  const float* cos_tab;
  const float* sin_tab;
  int rope_begin, rope_end;
  int rope_rows;  // rows of the cos / sin tables (positions must be below it)
  // SwiGLU: offset of the "up" half (rows of B in fwd, columns of gate|up in bwd)
  int pair_offset;
  // cross-entropy partials, [n_tiles, M]
  const int* labels;
  float* ce_max;  // [2 * n_tiles, M]
  float* ce_sum;
  int* ce_arg;
  float* ce_tgt;
  int* err;
  int stream_k;
  int splitk;  // EPI_F32ADD: > 1 selects K-chunk-major split-K instead of stream-K
  long splitk_slice;  // EPI_F32ADD: 0 = add into out (atomics); else split q stores into out + q * splitk_slice
  // fused-collective copy jobs, run by the epilogue warps before their first tile
  CopyJobs jobs;
};

struct TileSched {
  int m_tiles, n_tiles, nk;
  __device__ int tiles() const { return m_tiles * n_tiles; }
};

// Iterate the (tile, kb0, kb1) segments this CTA owns; identical in every role.
// mode 0: whole tiles strided over CTAs; 1: stream-K (even split of all k-blocks over CTAs);
// 2: fixed split-K (each tile in `split` equal k ranges; units ordered K chunk first).
template <typename F>
__device__ __forceinline__ void for_each_segment(const TileSched& s, int mode, int split, int unit, int units, F&& f) {
  const int total_tiles = s.tiles();
  if (mode == 0) {
    for (int t = unit; t < total_tiles; t += units) {
      if (!f(t, 0, s.nk)) return;
    }
    return;
  }
  if (mode == 2) {
    // K-chunk-major: the units running at the same time share one K chunk of both operands,
    // so that chunk stays in L2 instead of every tile streaming all of K from DRAM
    for (int u = unit; u < total_tiles * split; u += units) {
      const int q = u / total_tiles, t = u % total_tiles;
      const int kb0 = (int)((long long)s.nk * q / split), kb1 = (int)((long long)s.nk * (q + 1) / split);
      if (kb1 > kb0 && !f(t, kb0, kb1)) return;
    }
    return;
  }
  const long long total = (long long)total_tiles * s.nk;
  const long long begin = total * unit / units;
  const long long end = total * (unit + 1) / units;
  long long pos = begin;
  while (pos < end) {
    const int t = (int)(pos / s.nk);
    const int kb0 = (int)(pos % s.nk);
    const int kb1 = (int)min((long long)s.nk, kb0 + (end - pos));
    if (!f(t, kb0, kb1)) return;
    pos += kb1 - kb0;
  }
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Warp-uniform bounded spin until *p >= target (system-scope acquire by every lane).
__device__ __forceinline__ bool warp_wait_count_sys(const int* p, int target) {
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    if (__all_sync(0xffffffffu, ld_acquire_sys(p) >= target)) return true;
    if (__any_sync(0xffffffffu, globaltimer_ns() - t0 > kWaitTimeoutNs)) return false;
    __nanosleep(128);
  }
}
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
// smem tile -> global through a tensor map (the map's swizzle undoes the smem swizzle)
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(smem_u32(smem_src))
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// One epilogue warp's bf16 output path: lane = row of a 32-row box, w = its 32 columns as 16
// packed words. The box is written into one of the warp's two 2 KB buffers in the 64-byte
// swizzle of the output tensor map (16-byte piece q of row r at (q ^ (r / 2 % 4)) * 16, which
// keeps each quarter-warp's stores on distinct banks) and leaves with one TMA tensor store
// issued by lane 0; rows past the tensor's end are clipped by the map. A buffer is rewritten
// only after the store issued from it two boxes earlier has read it.
struct OutStager {
  uint8_t* base;
  int k;
  __device__ __forceinline__ void put(const CUtensorMap* map, const uint32_t (&w)[16], int lane, int x, int y) {
    uint8_t* buf = base + k * STG_BOX_BYTES;
    if (lane == 0) bulk_wait_read1();
    __syncwarp();
    const int sw = (lane >> 1) & 3;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *reinterpret_cast<uint4*>(buf + lane * 64 + ((q ^ sw) << 4)) =
          make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(map, buf, x, y);
      bulk_commit();
    }
    k ^= 1;
  }
};

__device__ __forceinline__ void pack_bf16x32(const float (&v)[32], uint32_t (&w)[16]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) w[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
}

// Bounded spin until *flag >= value (acquire); false after the time limit.
__device__ __forceinline__ bool wait_flag(const int* flag, int value) {
  if (ld_acquire_gpu(flag) >= value) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (ld_acquire_gpu(flag) < value) {
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) return false;
    __nanosleep(128);
  }
  return true;
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float (&v)[32]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w;
    w.x = pack_bf16x2(v[8 * q + 0], v[8 * q + 1]);
    w.y = pack_bf16x2(v[8 * q + 2], v[8 * q + 3]);
    w.z = pack_bf16x2(v[8 * q + 4], v[8 * q + 5]);
    w.w = pack_bf16x2(v[8 * q + 6], v[8 * q + 7]);
    d[q] = w;
  }
}

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* src, float (&v)[32]) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w = s[q];
    float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), c = unpack_bf16x2(w.z), d = unpack_bf16x2(w.w);
    v[8 * q + 0] = a.x; v[8 * q + 1] = a.y; v[8 * q + 2] = b.x; v[8 * q + 3] = b.y;
    v[8 * q + 4] = c.x; v[8 * q + 5] = c.y; v[8 * q + 6] = d.x; v[8 * q + 7] = d.y;
  }
}

__device__ __forceinline__ void tmem_load_f32x32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  tmem_ld_32x32b_x32(taddr, r);
  tmem_ld_wait();
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

template <int A_MN, int B_MN, int EPI, int PAIR = 0>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmC2,
                        const GemmArgs args) {
  constexpr int kStages = PAIR ? pair_stages<EPI>() : single_stages<EPI>();
  constexpr int kBStage = PAIR ? B_STAGE_BYTES / 2 : B_STAGE_BYTES;
  constexpr int TILE_M = PAIR ? 2 * BM : BM;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * A_STAGE_BYTES;
  uint8_t* sStage = sB + kStages * kBStage;  // 1024-aligned: stage sizes are multiples of 1 KB
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sStage + stage_bytes<EPI>());
  uint64_t* empty_bar = full_bar + kStages;
  uint64_t* tfull_bar = empty_bar + kStages;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint64_t* aux_bar = drain_bar + 1;  // SwiGLU backward: [epilogue warp][box pair] input loads
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aux_bar + 2 * EPI_WARPS);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // CTA pairs: rank 0 issues the UMMAs for both; each CTA owns rows [cta_rank*128, +128) of
  // the pair's 256-row tile. Work units are pairs.
  const uint32_t cta_rank = PAIR ? cluster_cta_rank() : 0u;
  const bool leader = cta_rank == 0;
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  TileSched sched;
  sched.m_tiles = (args.M + TILE_M - 1) / TILE_M;
  sched.n_tiles = (EPI == EPI_SWIGLU) ? (args.N + 127) / 128 : (args.N + BN - 1) / BN;
  sched.nk = (args.K + BK - 1) / BK;
  const int mode = (EPI == EPI_F32ADD && args.stream_k) ? (args.splitk > 1 ? 2 : 1) : 0;
  const int split = (mode == 2) ? args.splitk : 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      // pairs: lane 0 of every epilogue warp of both CTAs arrives on the leader's barrier
      mbar_init(&tempty_bar[a], PAIR ? 2 * EPI_WARPS : 32 * EPI_WARPS);
    }
    mbar_init(drain_bar, 1);
    for (int i = 0; i < 2 * EPI_WARPS; ++i) mbar_init(&aux_bar[i], 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    __syncwarp();
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();  // the peer's barriers are initialised
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      int issued_round[kStages];
#pragma unroll
      for (int s = 0; s < kStages; ++s) issued_round[s] = -1;
      bool ok = true;
      for_each_segment(sched, mode, split, unit, units, [&](int tile, int kb0, int kb1) -> bool {
        const int mt = tile / sched.n_tiles, nt = tile % sched.n_tiles;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % kStages, r = it / kStages;
          if (!mbar_wait(&empty_bar[s], (r & 1) ^ 1)) {
            report_error(args.err, kErrGemmWaitTimeout, 1);
            ok = false;
            return false;
          }
          uint8_t* a_dst = sA + s * A_STAGE_BYTES;
          uint8_t* b_dst = sB + s * kBStage;
          if constexpr (PAIR) {
            // both CTAs' copies complete on the leader's barrier, which expects all of them
            if (leader) mbar_arrive_expect_tx(&full_bar[s], 2 * (A_STAGE_BYTES + kBStage));
            const uint32_t fb = cluster_map(&full_bar[s], 0);
            const int row_a = mt * TILE_M + (int)cta_rank * BM;
            if (!A_MN) {
              tma_load_2d_pair(a_dst, &tmA, fb, kb * BK, row_a);
            } else {
              tma_load_2d_pair(a_dst, &tmA, fb, row_a, kb * BK);
              tma_load_2d_pair(a_dst + 8192, &tmA, fb, row_a + 64, kb * BK);
            }
            if (!B_MN) {  // this CTA's 128 columns of the tile: gate (rank 0) / up (rank 1) for SwiGLU
              const int rb = (EPI == EPI_SWIGLU) ? (cta_rank ? args.pair_offset + nt * 128 : nt * 128)
                                                 : nt * BN + (int)cta_rank * 128;
              tma_load_2d_pair(b_dst, &tmB, fb, kb * BK, rb);
            } else {
#pragma unroll
              for (int j = 0; j < 2; ++j)
                tma_load_2d_pair(b_dst + j * 8192, &tmB, fb, nt * BN + ((int)cta_rank * 2 + j) * 64, kb * BK);
            }
            issued_round[s] = r;
            continue;
          }
          mbar_arrive_expect_tx(&full_bar[s], A_STAGE_BYTES + B_STAGE_BYTES);
          if (!A_MN) {
            tma_load_2d(a_dst, &tmA, &full_bar[s], kb * BK, mt * BM);
          } else {
            tma_load_2d(a_dst, &tmA, &full_bar[s], mt * BM, kb * BK);
            tma_load_2d(a_dst + 8192, &tmA, &full_bar[s], mt * BM + 64, kb * BK);
          }
          if (!B_MN) {
            int r0, r1;
            if (EPI == EPI_SWIGLU) {
              r0 = nt * 128;
              r1 = args.pair_offset + nt * 128;
            } else {
              r0 = nt * BN;
              r1 = nt * BN + 128;
            }
            tma_load_2d(b_dst, &tmB, &full_bar[s], kb * BK, r0);
            tma_load_2d(b_dst + 16384, &tmB, &full_bar[s], kb * BK, r1);
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) tma_load_2d(b_dst + j * 8192, &tmB, &full_bar[s], nt * BN + j * 64, kb * BK);
          }
          issued_round[s] = r;
        }
        return true;
      });
      if (!ok && !PAIR) {
        // Drain: wait (bounded) until every load this thread issued has landed. (A pair's
        // copies complete on the leader's barriers; the closing cluster barrier covers them.)
        for (int s = 0; s < kStages; ++s)
          if (issued_round[s] >= 0) mbar_wait(&full_bar[s], issued_round[s] & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ UMMA issuer
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = umma_idesc_bf16(TILE_M, BN, A_MN, B_MN);
      int it = 0, local = 0;
      for_each_segment(sched, mode, split, unit, units, [&](int tile, int kb0, int kb1) -> bool {
        const int acc = local & 1, use = local >> 1;
        if (!mbar_wait(&tempty_bar[acc], (use & 1) ^ 1)) {
          report_error(args.err, kErrGemmWaitTimeout, 2);
          return false;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % kStages, r = it / kStages;
          if (!mbar_wait(&full_bar[s], r & 1)) {
            report_error(args.err, kErrGemmWaitTimeout, 3);
            return false;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + s * A_STAGE_BYTES);
          const uint32_t b_base = smem_u32(sB + s * kBStage);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = A_MN ? umma_desc_sw128(a_base + k * 2048, 8192, 1024)
                                        : umma_desc_sw128(a_base + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? umma_desc_sw128(b_base + k * 2048, 8192, 1024)
                                        : umma_desc_sw128(b_base + k * 32, 16, 1024);
            if constexpr (PAIR)
              umma_f16_ss_pair(d_tmem, adesc, bdesc, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
            else
              umma_f16_ss(d_tmem, adesc, bdesc, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          if constexpr (PAIR) {
            umma_commit_pair_mc(&empty_bar[s], 3);  // frees this stage in both CTAs
            continue;
          }
          umma_commit(&empty_bar[s]);  // frees the smem stage when these UMMAs finish
        }
        if constexpr (PAIR)
          umma_commit_pair_mc(&tfull_bar[acc], 3);  // both CTAs' accumulator halves ready
        else
          umma_commit(&tfull_bar[acc]);  // accumulator ready for the epilogue
        ++local;
        return true;
      });
      // Make sure every UMMA this thread issued has completed before TMEM is released.
      if constexpr (PAIR)
        umma_commit_pair_mc(drain_bar, 1);
      else
        umma_commit(drain_bar);
      mbar_wait(drain_bar, 0);
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;  // which column half of the tile this warp handles
    const int row = quarter * 32 + lane;
    if (args.jobs.g_src != nullptr || args.jobs.p_src != nullptr)
      run_copy_jobs(args.jobs, (int)blockIdx.x * EPI_WARPS + (warp - 2), (int)gridDim.x * EPI_WARPS, lane);
    OutStager stg{sStage + (warp - 2) * 2 * STG_BOX_BYTES, 0};
    // SwiGLU backward: this warp's two (g | u) box pairs, and the chunk stream they are loaded for
    uint8_t* aux_base = sStage + (warp - 2) * 4 * STG_BOX_BYTES;
    uint64_t* my_aux_bar = aux_bar + 2 * (warp - 2);
    int aux_j = 0;           // chunks of this warp consumed so far (pair = j & 1, phase = (j >> 1) & 1)
    int aux_loaded = 0;      // chunks whose loads were issued
    // lane 0: g and u boxes of chunk (mt, nt, c) into pair p
    auto aux_issue = [&](int p, int lmt, int lnt, int c) {
      if (lane == 0) {
        uint8_t* b = aux_base + p * 2 * STG_BOX_BYTES;
        const int y = lmt * TILE_M + (int)cta_rank * BM + quarter * 32;
        const int f = lnt * BN + c * 32;
        mbar_arrive_expect_tx(&my_aux_bar[p], 2 * STG_BOX_BYTES);
        tma_load_2d(b, &tmC2, &my_aux_bar[p], f, y);
        tma_load_2d(b + STG_BOX_BYTES, &tmC2, &my_aux_bar[p], args.pair_offset + f, y);
      }
    };
    int local = 0;
    for_each_segment(sched, mode, split, unit, units, [&](int tile, int kb0, int kb1) -> bool {
      const int mt = tile / sched.n_tiles, nt = tile % sched.n_tiles;
      const int acc = local & 1, use = local >> 1;
      // warp-uniform outcome: the TMEM loads below are warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull_bar[acc], use & 1))) {
        report_error(args.err, kErrGemmWaitTimeout, 4);
        return false;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      const int m = mt * TILE_M + (int)cta_rank * BM + row;
      const bool row_ok = m < args.M;
      const int box_y = mt * TILE_M + (int)cta_rank * BM + quarter * 32;  // this warp's 32 rows

      if constexpr (EPI == EPI_STORE) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = half * 4 + q;
          float v[32];
          tmem_load_f32x32(taddr + c * 32, v);
          const int n = nt * BN + c * 32;
          if (n < args.N) {  // warp-uniform; rows past M are clipped by the store
            uint32_t w[16];
            pack_bf16x32(v, w);
            stg.put(&tmC, w, lane, n, box_y);
          }
        }
      } else if constexpr (EPI == EPI_RESIDUAL) {
        // The residual arrives as 32 x 32 TMA boxes in this warp's two buffers (the next chunk's
        // load, also across tiles, is issued before this chunk is computed); the sum is written
        // over it in place and leaves through a TMA store. Rows past M load as zeros and their
        // stores are clipped; the output may alias the residual (each box is read, then written).
        uint8_t* res_base = sStage + (warp - 2) * 2 * STG_BOX_BYTES;
        auto res_issue = [&](int p, int lmt, int lnt, int c) {
          if (lane == 0) {
            mbar_arrive_expect_tx(&my_aux_bar[p], STG_BOX_BYTES);
            tma_load_2d(res_base + p * STG_BOX_BYTES, &tmC2, &my_aux_bar[p], lnt * BN + c * 32,
                        lmt * TILE_M + (int)cta_rank * BM + quarter * 32);
          }
        };
        const int next_tile = tile + units;  // whole-tile schedule: this warp's next tile
        if (aux_loaded == aux_j) {           // nothing in flight (first tile of the warp)
          res_issue(aux_j & 1, mt, nt, half * 4);
          ++aux_loaded;
        }
#pragma unroll 1
        for (int q = 0; q < 4; ++q) {
          const int c = half * 4 + q;
          const int n = nt * BN + c * 32;
          const int p = aux_j & 1;
          if (q < 3 || next_tile < sched.tiles()) {
            if (lane == 0) bulk_wait_read0();  // the previous chunk's store has read the other buffer
            __syncwarp();
            const int nmt = q < 3 ? mt : next_tile / sched.n_tiles, nnt = q < 3 ? nt : next_tile % sched.n_tiles;
            res_issue(p ^ 1, nmt, nnt, q < 3 ? c + 1 : half * 4);
            ++aux_loaded;
          }
          float v[32];
          tmem_load_f32x32(taddr + c * 32, v);
          if (!__all_sync(0xffffffffu, mbar_wait(&my_aux_bar[p], (aux_j >> 1) & 1))) {
            report_error(args.err, kErrGemmWaitTimeout, 7);
            return false;
          }
          uint8_t* rb = res_base + p * STG_BOX_BYTES;
          const int sw = (lane >> 1) & 3;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4* rp = reinterpret_cast<uint4*>(rb + lane * 64 + ((i ^ sw) << 4));
            const uint4 w = *rp;
            const float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), cc = unpack_bf16x2(w.z),
                         d = unpack_bf16x2(w.w);
            *rp = make_uint4(pack_bf16x2(v[8 * i + 0] + a.x, v[8 * i + 1] + a.y),
                             pack_bf16x2(v[8 * i + 2] + b.x, v[8 * i + 3] + b.y),
                             pack_bf16x2(v[8 * i + 4] + cc.x, v[8 * i + 5] + cc.y),
                             pack_bf16x2(v[8 * i + 6] + d.x, v[8 * i + 7] + d.y));
          }
          fence_async_smem();
          __syncwarp();
          if (n < args.N && lane == 0) tma_store_2d(&tmC, rb, n, box_y);  // warp-uniform column bound
          if (lane == 0) bulk_commit();
          ++aux_j;
        }
      } else if constexpr (EPI == EPI_F32ADD) {
        float* out = reinterpret_cast<float*>(args.out);
        // deterministic split-K: the unit of K chunk q stores its partial into slice q (the
        // caller sums the slices in order); kb0 = floor(nk * q / split) identifies q
        const bool sliced = args.splitk_slice != 0;
        if (sliced) out += (long)((mode == 2) ? (kb0 * split + sched.nk - 1) / sched.nk : 0) * args.splitk_slice;
#pragma unroll 1
        for (int c = half * 4; c < half * 4 + 4; ++c) {
          float v[32];
          tmem_load_f32x32(taddr + c * 32, v);
          const int n = nt * BN + c * 32;
          if (row_ok && n < args.N) {
            float4* dst = reinterpret_cast<float4*>(out + (long)m * args.ldo + n);
            if (sliced) {
#pragma unroll
              for (int q = 0; q < 8; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            } else {
#pragma unroll
              for (int q = 0; q < 8; ++q)
                atomicAdd(dst + q, make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
            }
          }
        }
      } else if constexpr (EPI == EPI_ROPE) {
        // This warp handles frequency chunk c = half (columns [c*32, c*32+32) paired with +64)
        // of both 128-wide heads of the tile, 16 frequencies at a time (the cos / sin slices are
        // re-read per head from L1) so the live registers stay under the 320-thread cap.
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(args.out);
        const int c = half;
        int pos = row_ok ? args.positions[m] : 0;
        if (!HRM_BOUNDS_OK(pos >= 0 && pos < args.rope_rows, args.err, 80)) pos = 0;
        const float4* cr = reinterpret_cast<const float4*>(args.cos_tab + (long)pos * 64 + c * 32);
        const float4* sr = reinterpret_cast<const float4*>(args.sin_tab + (long)pos * 64 + c * 32);
        // this row's 32 frequencies of the chunk, read once and used for both heads of the tile
        const bool any_rotate = (nt * BN < args.rope_end) && (nt * BN + 256 > args.rope_begin);
        float cs_all[32], sn_all[32];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 a = (row_ok && any_rotate) ? cr[q] : make_float4(0.f, 0.f, 0.f, 0.f);
          const float4 b = (row_ok && any_rotate) ? sr[q] : make_float4(0.f, 0.f, 0.f, 0.f);
          cs_all[4 * q] = a.x; cs_all[4 * q + 1] = a.y; cs_all[4 * q + 2] = a.z; cs_all[4 * q + 3] = a.w;
          sn_all[4 * q] = b.x; sn_all[4 * q + 1] = b.y; sn_all[4 * q + 2] = b.z; sn_all[4 * q + 3] = b.w;
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int head_col = nt * BN + h * 128;
          const bool rotate = head_col >= args.rope_begin && head_col < args.rope_end;
          uint32_t o1[16], o2[16];  // columns head_col + c*32 + [0,32) and head_col + 64 + c*32 + [0,32)
#pragma unroll
          for (int sub = 0; sub < 2; ++sub) {
            uint32_t r1[16], r2[16];
            tmem_ld_32x32b_x16(taddr + h * 128 + c * 32 + sub * 16, r1);
            tmem_ld_32x32b_x16(taddr + h * 128 + 64 + c * 32 + sub * 16, r2);
            const float* cs = cs_all + sub * 16;
            const float* sn = sn_all + sub * 16;
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
              float a0 = __uint_as_float(r1[j]), a1 = __uint_as_float(r1[j + 1]);
              float b0 = __uint_as_float(r2[j]), b1 = __uint_as_float(r2[j + 1]);
              if (rotate) {
                const float na0 = a0 * cs[j] - b0 * sn[j], na1 = a1 * cs[j + 1] - b1 * sn[j + 1];
                const float nb0 = b0 * cs[j] + a0 * sn[j], nb1 = b1 * cs[j + 1] + a1 * sn[j + 1];
                a0 = na0; a1 = na1; b0 = nb0; b1 = nb1;
              }
              o1[sub * 8 + (j >> 1)] = pack_bf16x2(a0, a1);
              o2[sub * 8 + (j >> 1)] = pack_bf16x2(b0, b1);
            }
          }
          if (head_col < args.N) {  // warp-uniform
            stg.put(&tmC, o1, lane, head_col + c * 32, box_y);
            stg.put(&tmC, o2, lane, head_col + 64 + c * 32, box_y);
          }
        }
        (void)out;
      } else if constexpr (EPI == EPI_SWIGLU) {
        // acc columns [0,128) = gate, [128,256) = up for features nt*128 + [0,128)
        __nv_bfloat16* gu = reinterpret_cast<__nv_bfloat16*>(args.out);
        __nv_bfloat16* hout = reinterpret_cast<__nv_bfloat16*>(args.out2);
#pragma unroll 1
        for (int c = half * 2; c < half * 2 + 2; ++c) {
          float g[32], u[32];
          tmem_load_f32x32(taddr + c * 32, g);
          tmem_load_f32x32(taddr + 128 + c * 32, u);
          const int f = nt * 128 + c * 32;
          if (f < args.N) {  // warp-uniform
            float hv[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              g[j] = bf16_round(g[j]);
              u[j] = bf16_round(u[j]);
              hv[j] = __fdividef(g[j], 1.0f + __expf(-g[j])) * u[j];  // fast divide: output is bf16
            }
            uint32_t w[16];
            pack_bf16x32(g, w);
            stg.put(&tmC, w, lane, f, box_y);
            pack_bf16x32(u, w);
            stg.put(&tmC, w, lane, args.pair_offset + f, box_y);
            pack_bf16x32(hv, w);
            stg.put(&tmC2, w, lane, f, box_y);
          }
        }
        (void)gu; (void)hout;
      } else if constexpr (EPI == EPI_SWIGLU_BWD) {
        // g / u arrive as 32 x 32 TMA boxes in this warp's buffers (loads for the next chunk,
        // also across tiles, are issued before this chunk is computed); d(gate) / d(up) are
        // written over them in place and leave through TMA stores. Rows past M load as zeros
        // and their stores are clipped.
        const int next_tile = tile + units;  // whole-tile schedule: this warp's next tile
        if (aux_loaded == aux_j) {           // nothing in flight (first tile of the warp)
          aux_issue(aux_j & 1, mt, nt, half * 4);
          ++aux_loaded;
        }
#pragma unroll 1
        for (int q = 0; q < 4; ++q) {
          const int c = half * 4 + q;
          const int f = nt * BN + c * 32;
          const int p = aux_j & 1;
          // the other pair held the previous chunk: its stores must have read it before reuse
          const bool more = q < 3 || next_tile < sched.tiles();
          if (more) {
            if (lane == 0) bulk_wait_read0();
            __syncwarp();
            const int nq = q < 3 ? q + 1 : 0;
            const int nmt = q < 3 ? mt : next_tile / sched.n_tiles, nnt = q < 3 ? nt : next_tile % sched.n_tiles;
            aux_issue(p ^ 1, nmt, nnt, half * 4 + nq);
            ++aux_loaded;
          }
          float dh[32];
          tmem_load_f32x32(taddr + c * 32, dh);
          if (!__all_sync(0xffffffffu, mbar_wait(&my_aux_bar[p], (aux_j >> 1) & 1))) {
            report_error(args.err, kErrGemmWaitTimeout, 6);
            return false;
          }
          uint8_t* gb = aux_base + p * 2 * STG_BOX_BYTES;
          uint8_t* ub = gb + STG_BOX_BYTES;
          const int sw = (lane >> 1) & 3;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4* gp = reinterpret_cast<uint4*>(gb + lane * 64 + ((i ^ sw) << 4));
            uint4* up = reinterpret_cast<uint4*>(ub + lane * 64 + ((i ^ sw) << 4));
            const uint4 gw4 = *gp, uw4 = *up;
            const uint32_t gw[4] = {gw4.x, gw4.y, gw4.z, gw4.w};
            const uint32_t uw[4] = {uw4.x, uw4.y, uw4.z, uw4.w};
            uint32_t dgw[4], duw[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float2 g2 = unpack_bf16x2(gw[k]), u2 = unpack_bf16x2(uw[k]);
              float o_g[2], o_u[2];
              const float gv[2] = {g2.x, g2.y}, uv[2] = {u2.x, u2.y};
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const float sg = __fdividef(1.0f, 1.0f + __expf(-gv[e]));  // fast divide: outputs are bf16
                const float silu = gv[e] * sg;
                const float dsilu = sg * (1.0f + gv[e] * (1.0f - sg));
                const float d = bf16_round(dh[8 * i + 2 * k + e]);
                o_g[e] = d * uv[e] * dsilu;
                o_u[e] = d * silu;
              }
              dgw[k] = pack_bf16x2(o_g[0], o_g[1]);
              duw[k] = pack_bf16x2(o_u[0], o_u[1]);
            }
            *gp = make_uint4(dgw[0], dgw[1], dgw[2], dgw[3]);
            *up = make_uint4(duw[0], duw[1], duw[2], duw[3]);
          }
          fence_async_smem();
          __syncwarp();
          if (f < args.N && lane == 0) {  // warp-uniform column bound
            const int y = mt * TILE_M + (int)cta_rank * BM + quarter * 32;
            tma_store_2d(&tmC, gb, f, y);
            tma_store_2d(&tmC, ub, args.pair_offset + f, y);
          }
          if (lane == 0) bulk_commit();
          ++aux_j;
        }
      } else if constexpr (EPI == EPI_CE_BWD) {
        // Logits of one V chunk (columns [col0, col0 + N) of the head), recomputed by this GEMM
        // and rounded to bf16 exactly as the forward's statistics saw them, turned into
        // (softmax - onehot) * dloss with the forward's log-sum-exp; rows without a label are 0.
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(args.out);
        const int label = row_ok ? args.labels[m] : -1;
        const float lse = row_ok ? args.ce_max[m] : 0.f;  // natural-log LSE per row
        const float g = *args.ce_sum;                     // d loss_sum
        const int col0 = args.pair_offset;
#pragma unroll 1
        for (int c = half * 4; c < half * 4 + 4; ++c) {
          float v[32];
          tmem_load_f32x32(taddr + c * 32, v);
          const int n = nt * BN + c * 32;
          if (n < args.N) {  // warp-uniform; rows past M are clipped by the store
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float prob = __expf(bf16_round(v[j]) - lse);
              v[j] = label < 0 ? 0.f : (prob - (col0 + n + j == label ? 1.f : 0.f)) * g;
            }
            uint32_t w[16];
            pack_bf16x32(v, w);
            stg.put(&tmC, w, lane, n, box_y);
          }
        }
        (void)out;
      } else if constexpr (EPI == EPI_CE) {
        // Partial softmax statistics over this warp's 128 columns; partial index nt*2 + half.
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(args.out);
        const int label = row_ok ? args.labels[m] : -1;
        float run_max = -INFINITY, run_sum = 0.0f;
        int run_arg = 0;
        constexpr float kLog2e = 1.4426950408889634f;
#pragma unroll 1
        for (int c = half * 4; c < half * 4 + 4; ++c) {
          float v[32];
          tmem_load_f32x32(taddr + c * 32, v);
          const int n = nt * BN + c * 32;
          if (row_ok && n < args.N) {
            float cmax = -INFINITY;
            int carg = 0;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              v[j] = bf16_round(v[j]);
              if (v[j] > cmax) {
                cmax = v[j];
                carg = j;
              }
              if (n + j == label) args.ce_tgt[m] = v[j];
            }
            const float new_max = fmaxf(run_max, cmax);
            float s = 0.0f;
#pragma unroll
            for (int j = 0; j < 32; ++j) s += fast_exp2((v[j] - new_max) * kLog2e);
            run_sum = run_sum * fast_exp2((run_max - new_max) * kLog2e) + s;
            if (cmax > run_max) run_arg = n + carg;
            run_max = new_max;
            if (out != nullptr) store_bf16x32(out + (long)m * args.ldo + n, v);  // null: statistics only
          }
        }
        if (row_ok) {
          const long idx = (long)(nt * 2 + half) * args.M + m;
          args.ce_max[idx] = run_max;
          args.ce_sum[idx] = run_sum;
          args.ce_arg[idx] = run_arg;
        }
      }
      tc_fence_before();
      if constexpr (PAIR) {
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(cluster_map(&tempty_bar[acc], 0));
      } else {
        mbar_arrive(&tempty_bar[acc]);
      }
      ++local;
      return true;
    });
    if constexpr (EPI == EPI_SWIGLU_BWD || EPI == EPI_RESIDUAL) {
      // loads issued for chunks that were never consumed (a wait gave up): let them land
      for (int jj = aux_j; jj < aux_loaded; ++jj) mbar_wait(&my_aux_bar[jj & 1], (jj >> 1) & 1);
    }
  }

  if (warp >= 2 && lane == 0) bulk_wait0();  // this warp's output stores are complete
  tc_fence_before();
  __syncthreads();
  // pairs: the leader's UMMAs write the peer's TMEM and read its shared memory, and its commits
  // arrive there: neither CTA releases TMEM or exits before both are done
  if constexpr (PAIR) cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else
      tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

// 2D bf16 tensor map over a row-major matrix [outer, inner] with row stride `ld` elements.
CUtensorMap make_map(const at::Tensor& t, int64_t inner, int64_t outer, int64_t ld, uint32_t box_inner,
                     uint32_t box_outer) {
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, "GEMM operands must be bf16");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, "GEMM operand base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "GEMM operand row stride must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, t.data_ptr(), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", (int)r);
  return map;
}

// bf16 output tensor [rows, t.size(1)] (row stride t.stride(0)) as 32 x 32 boxes in the 64-byte
// swizzle that OutStager writes.
CUtensorMap make_out_map(const at::Tensor& t, int64_t rows) {
  TORCH_CHECK(t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.stride(1) == 1, "GEMM output must be row-major bf16");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0 && (t.stride(0) * 2) % 16 == 0,
              "GEMM output base and row stride must be 16-byte aligned");
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)t.size(1), (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(t.stride(0) * 2)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, t.data_ptr(), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (output) failed with code ", (int)r);
  return map;
}

int num_sms() { return device_sm_count(); }

// Split-K factor of an fp32 weight-gradient GEMM: at least `s0` (the split whose K-chunk operand
// panels stay L2-sized), up to 2*s0 + 2, minimising the estimated time of `tiles * s` units on
// `units` persistent CTA pairs: waves * (1/s + c), where c = 0.05 of a whole tile's main loop is
// the per-unit cost (epilogue, fp32 reductions, pipeline fill; fitted on the HRM-Text L weight
// gradients). It changes only GEMMs whose units quantise badly: the L o_proj gradient
// (25 tiles x 3 units on 74 pairs: two waves for one wave's work) went from 0.107 to 0.064 ms.
int balanced_split(int s0, int64_t tiles, int units, int64_t nk) {
  if (s0 <= 1 || units <= 0) return s0;
  auto cost = [&](int s) { return (double)((tiles * s + units - 1) / units) * (1.0 / s + 0.05); };
  const int hi = (int)std::min<int64_t>(2 * s0 + 2, nk);
  double best = cost(s0);
  for (int s = s0 + 1; s <= hi; ++s) best = std::min(best, cost(s));
  for (int s = s0; s <= hi; ++s)
    if (cost(s) <= best * 1.02) return s;
  return s0;
}

// CTA pairs that can be resident at once (cluster placement can leave SMs unused).
template <int A_MN, int B_MN, int EPI>
int max_pair_clusters() {
  static std::atomic<int> per_device[kMaxDevices];  // per kernel instantiation and device
  const int dev = current_device();
  TORCH_CHECK(dev < kMaxDevices, "device index out of range");
  int n = per_device[dev].load(std::memory_order_acquire);
  if (n == 0) {
    auto kern = gemm_tcgen05_kernel<A_MN, B_MN, EPI, 1>;
    TORCH_CHECK(ensure_dynamic_smem((const void*)kern, pair_smem_bytes<EPI>()) == cudaSuccess,
                "cudaFuncSetAttribute failed");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (num_sms() / 2));
    cfg.blockDim = dim3(GEMM_THREADS);
    cfg.dynamicSmemBytes = pair_smem_bytes<EPI>();
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    TORCH_CHECK(cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) == cudaSuccess && clusters > 0,
                "no CTA pair of the GEMM fits on this device");
    n = std::min(clusters, num_sms() / 2);
    per_device[dev].store(n, std::memory_order_release);
  }
  return n;
}

template <int A_MN, int B_MN, int EPI>
void launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const CUtensorMap& mc2,
                 const GemmArgs& args, int clusters, cudaStream_t stream) {
  auto kern = gemm_tcgen05_kernel<A_MN, B_MN, EPI, 1>;
  max_pair_clusters<A_MN, B_MN, EPI>();  // sets the shared-memory attribute
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = pair_smem_bytes<EPI>();
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  TORCH_CHECK(cudaLaunchKernelEx(&cfg, kern, ma, mb, mc, mc2, args) == cudaSuccess, "pair GEMM launch failed");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int A_MN, int B_MN, int EPI>
void launch(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const CUtensorMap& mc2,
            const GemmArgs& args, int grid, cudaStream_t stream) {
  auto kern = gemm_tcgen05_kernel<A_MN, B_MN, EPI>;
  TORCH_CHECK(ensure_dynamic_smem((const void*)kern, gemm_smem_bytes<EPI>()) == cudaSuccess,
              "cudaFuncSetAttribute failed");
  kern<<<grid, GEMM_THREADS, gemm_smem_bytes<EPI>(), stream>>>(ma, mb, mc, mc2, args);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace

at::Tensor device_error_word();  // errors.cu
CopyJobs decode_copy_jobs(const at::Tensor& d);

// Generic entry: see the file header for operand conventions.
//   a: [M,K] (a_mn=0) or [K,M] (a_mn=1);  b: [Nb,K] (b_mn=0) or [K,N] (b_mn=1)
void gemm(const at::Tensor& a, bool a_mn, const at::Tensor& b, bool b_mn, int64_t M, int64_t N, int64_t K,
          int64_t epi, const at::Tensor& out, const c10::optional<at::Tensor>& out2,
          const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& aux,
          const c10::optional<at::Tensor>& positions, const c10::optional<at::Tensor>& cos_tab,
          const c10::optional<at::Tensor>& sin_tab, int64_t rope_begin, int64_t rope_end, int64_t pair_offset,
          const c10::optional<at::Tensor>& labels, const c10::optional<at::Tensor>& ce_max,
          const c10::optional<at::Tensor>& ce_sum, const c10::optional<at::Tensor>& ce_arg,
          const c10::optional<at::Tensor>& ce_tgt, bool stream_k, int64_t splitk,
          const c10::optional<at::Tensor>& jobs) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && out.is_cuda(), "gemm: CUDA tensors expected");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1, "gemm: row-major 2D operands");
  TORCH_CHECK(N % 32 == 0, "gemm: N must be a multiple of 32");
  c10::cuda::CUDAGuard guard(a.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();

  GemmArgs args{};
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  if (epi == EPI_CE && out.numel() == 0) {  // cross-entropy statistics without storing the logits
    args.out = nullptr;
    args.ldo = 0;
  } else if (epi == EPI_F32ADD && out.dim() == 3) {  // deterministic split-K: [split, M, N] fp32 slices
    TORCH_CHECK(out.stride(2) == 1 && out.stride(1) % 4 == 0 && out.size(1) == M && out.size(2) == N &&
                    out.size(0) >= 1 && out.size(0) <= (K + BK - 1) / BK,
                "gemm: split-K slices must be [split <= k-blocks, M, N] fp32 with 16-byte aligned rows");
    args.out = out.data_ptr();
    args.ldo = out.stride(1);
    args.splitk_slice = out.stride(0);
    splitk = out.size(0);
    stream_k = splitk > 1;  // one slice: whole tiles, plain stores
  } else {
    args.out = out.data_ptr();
    args.ldo = out.stride(0);
    TORCH_CHECK(out.stride(1) == 1 && out.stride(0) % 8 == 0, "gemm: output rows must be contiguous and 16B aligned");
  }
  if (out2) { args.out2 = out2->data_ptr(); args.ldo2 = out2->stride(0); }
  if (residual) { args.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()); args.ldr = residual->stride(0); }
  if (aux) { args.aux = reinterpret_cast<const __nv_bfloat16*>(aux->data_ptr()); args.ldaux = aux->stride(0); }
  if (positions) args.positions = positions->data_ptr<int>();
  if (cos_tab) {
    args.cos_tab = cos_tab->data_ptr<float>();
    args.rope_rows = (int)cos_tab->size(0);
  }
  if (sin_tab) args.sin_tab = sin_tab->data_ptr<float>();
  args.rope_begin = (int)rope_begin;
  args.rope_end = (int)rope_end;
  args.pair_offset = (int)pair_offset;
  if (labels) args.labels = labels->data_ptr<int>();
  if (ce_max) args.ce_max = ce_max->data_ptr<float>();
  if (ce_sum) args.ce_sum = ce_sum->data_ptr<float>();
  if (ce_arg) args.ce_arg = ce_arg->data_ptr<int>();
  if (ce_tgt) args.ce_tgt = ce_tgt->data_ptr<float>();
  args.err = device_error_word().data_ptr<int>();
  if (jobs) args.jobs = decode_copy_jobs(*jobs);
  args.stream_k = stream_k ? 1 : 0;
  // fp32 weight gradients with a long K (tokens): split K into chunks whose operand slices
  // (both [chunk, M] and [chunk, N] panels, ~48 MB) fit in L2 next to the accumulation traffic
  args.splitk = 1;
  if (epi == EPI_F32ADD && stream_k) {
    const double panel_bytes = 2.0 * (double)K * (double)(M + N);
    // operand bytes per K chunk, HRM_WGRAD_PANEL_MB (default 72 MB: at L, 48 / 72 / 96 MB measured
    // gate/up 0.373 / 0.315 / 0.309 ms, qkv 0.231 / 0.224 / 0.229 ms, down 0.156 / 0.151 / 0.151)
    static const double panel_target = [] {
      const char* v = std::getenv("HRM_WGRAD_PANEL_MB");
      return (v != nullptr && std::atof(v) > 0.0) ? std::atof(v) * 1024.0 * 1024.0 : 72.0 * 1024.0 * 1024.0;
    }();
    args.splitk = (int)std::min<double>(16.0, std::max(1.0, std::ceil(panel_bytes / panel_target)));
    static const bool chunked = [] {
      const char* v = std::getenv("HRM_WGRAD_SPLITK");
      return v == nullptr || std::string(v) != "0";
    }();
    if (!chunked) args.splitk = 1;
    // an explicit split (decode-step GEMMs: a few rows, K spread over many CTAs)
    if (splitk > 0) args.splitk = (int)std::max<int64_t>(1, std::min<int64_t>(splitk, (K + BK - 1) / BK));
  }

  CUtensorMap ma = a_mn ? make_map(a, M, K, a.stride(0), 64, 64) : make_map(a, K, M, a.stride(0), 64, 128);
  const int64_t b_rows = b_mn ? K : b.size(0);
  CUtensorMap mb = b_mn ? make_map(b, N, K, b.stride(0), 64, 64) : make_map(b, K, b_rows, b.stride(0), 64, 128);
  // bf16 outputs leave through TMA stores (OutStager); other epilogues get unused placeholders
  CUtensorMap mc = ma, mc2 = ma;
  if (epi == EPI_STORE || epi == EPI_RESIDUAL || epi == EPI_ROPE || epi == EPI_SWIGLU || epi == EPI_SWIGLU_BWD ||
      epi == EPI_CE_BWD) {
    mc = make_out_map(out, M);
    if (epi == EPI_SWIGLU) {
      TORCH_CHECK(out2.has_value(), "gemm: the SwiGLU epilogue needs its second output");
      mc2 = make_out_map(*out2, M);
    }
    if (epi == EPI_RESIDUAL) {  // the residual, loaded as boxes of the output's shape
      TORCH_CHECK(residual.has_value(), "gemm: the residual epilogue needs its residual");
      mc2 = make_out_map(*residual, M);
    }
    if (epi == EPI_SWIGLU_BWD) {  // g | u inputs, loaded as boxes of the same shape
      TORCH_CHECK(aux.has_value() && aux->size(1) >= 2 * pair_offset, "gemm: the SwiGLU backward needs g | u");
      mc2 = make_out_map(*aux, M);
    }
  }

  const int64_t n_tiles = (epi == EPI_SWIGLU) ? (N + 127) / 128 : (N + BN - 1) / BN;
  // CTA pairs (256-row tiles) unless the problem is too short to fill them
  static const bool pair_enabled = [] {
    const char* v = std::getenv("HRM_GEMM_PAIR");
    return v == nullptr || std::string(v) != "0";
  }();
  const bool pair = pair_enabled && M >= 1024;
  if (pair) {
    const int64_t tiles = ((M + 2 * BM - 1) / (2 * BM)) * n_tiles;
    static const bool balance = [] {  // HRM_WGRAD_BALANCE=0: the plain L2-sized split (A/B runs)
      const char* v = std::getenv("HRM_WGRAD_BALANCE");
      return v == nullptr || std::string(v) != "0";
    }();
    if (balance && epi == EPI_F32ADD && stream_k && splitk <= 0 && args.splitk > 1)  // automatic split only
      args.splitk = balanced_split(args.splitk, tiles, max_pair_clusters<1, 1, EPI_F32ADD>(), (K + BK - 1) / BK);
#define HRM_GEMM_PAIR_CASE(AM, BMJ, E)                                                             \
  if (a_mn == AM && b_mn == BMJ && epi == E) {                                                     \
    const int cl = max_pair_clusters<AM, BMJ, E>();                                                \
    const int clusters = (E == EPI_F32ADD && stream_k) ? cl : (int)std::min<int64_t>(tiles, cl);   \
    return launch_pair<AM, BMJ, E>(ma, mb, mc, mc2, args, clusters, stream);                      \
  }
    HRM_GEMM_PAIR_CASE(0, 0, EPI_STORE)
    HRM_GEMM_PAIR_CASE(0, 0, EPI_RESIDUAL)
    HRM_GEMM_PAIR_CASE(0, 0, EPI_ROPE)
    HRM_GEMM_PAIR_CASE(0, 0, EPI_SWIGLU)
    HRM_GEMM_PAIR_CASE(0, 0, EPI_CE)
    HRM_GEMM_PAIR_CASE(0, 0, EPI_F32ADD)
    HRM_GEMM_PAIR_CASE(0, 0, EPI_CE_BWD)
    HRM_GEMM_PAIR_CASE(0, 1, EPI_F32ADD)
    HRM_GEMM_PAIR_CASE(0, 1, EPI_STORE)
    HRM_GEMM_PAIR_CASE(0, 1, EPI_RESIDUAL)
    HRM_GEMM_PAIR_CASE(0, 1, EPI_SWIGLU_BWD)
    HRM_GEMM_PAIR_CASE(1, 1, EPI_F32ADD)
    HRM_GEMM_PAIR_CASE(1, 1, EPI_STORE)
#undef HRM_GEMM_PAIR_CASE
  }
  const int64_t m_tiles = (M + BM - 1) / BM;
  const int64_t tiles = m_tiles * n_tiles;
  int grid = (int)std::min<int64_t>(tiles, num_sms());
  if (epi == EPI_F32ADD && stream_k) grid = num_sms();

#define HRM_GEMM_CASE(AM, BMJ, E) \
  if (a_mn == AM && b_mn == BMJ && epi == E) return launch<AM, BMJ, E>(ma, mb, mc, mc2, args, grid, stream);
  HRM_GEMM_CASE(0, 0, EPI_STORE)
  HRM_GEMM_CASE(0, 0, EPI_RESIDUAL)
  HRM_GEMM_CASE(0, 0, EPI_ROPE)
  HRM_GEMM_CASE(0, 0, EPI_SWIGLU)
  HRM_GEMM_CASE(0, 0, EPI_CE)
  HRM_GEMM_CASE(0, 0, EPI_F32ADD)
  HRM_GEMM_CASE(0, 0, EPI_CE_BWD)
  HRM_GEMM_CASE(0, 1, EPI_F32ADD)
  HRM_GEMM_CASE(0, 1, EPI_STORE)
  HRM_GEMM_CASE(0, 1, EPI_RESIDUAL)
  HRM_GEMM_CASE(0, 1, EPI_SWIGLU_BWD)
  HRM_GEMM_CASE(1, 1, EPI_F32ADD)
  HRM_GEMM_CASE(1, 1, EPI_STORE)
#undef HRM_GEMM_CASE
  TORCH_CHECK(false, "gemm: unsupported (a_mn, b_mn, epilogue) combination ", a_mn, b_mn, epi);
}

// The weight-gradient split choice on its own (host arithmetic, no device needed): for tests
// and for tools that plan launches.
int64_t gemm_balanced_split(int64_t s0, int64_t tiles, int64_t units, int64_t nk) {
  return balanced_split((int)s0, tiles, (int)units, nk);
}

// Fused-collective copy jobs for one launch (collective_jobs.cuh), from a CPU int64 [16]
// descriptor: {gather: src addresses tensor ptr, dst ptr, rows, cols, rows per rank;
// push: src ptr, base addresses tensor ptr, inbox offset, inbox slot stride, count offset,
// rows, cols, rows per rank, rank, ran-flag ptr; unused}. Addresses are device pointers.
CopyJobs decode_copy_jobs(const at::Tensor& d) {
  TORCH_CHECK(!d.is_cuda() && d.scalar_type() == at::kLong && d.numel() == 16, "copy jobs: CPU int64 [16] expected");
  const int64_t* v = d.data_ptr<int64_t>();
  CopyJobs j{};
  if (v[0] != 0) {
    j.g_src = reinterpret_cast<const unsigned long long*>(v[0]);
    j.g_dst = reinterpret_cast<__nv_bfloat16*>(v[1]);
    j.g_rows = (int)v[2]; j.g_cols = (int)v[3]; j.g_chunk = (int)v[4];
    TORCH_CHECK(j.g_cols % 8 == 0 && j.g_chunk > 0 && (v[1] & 15) == 0, "gather job: 16-byte aligned rows expected");
  }
  if (v[5] != 0) {
    j.p_src = reinterpret_cast<const float*>(v[5]);
    j.p_base = reinterpret_cast<const unsigned long long*>(v[6]);
    j.p_inbox_off = v[7]; j.p_inbox_stride = v[8]; j.p_cnt_off = v[9];
    j.p_rows = (int)v[10]; j.p_cols = (int)v[11]; j.p_chunk = (int)v[12]; j.p_rank = (int)v[13];
    j.p_ran = reinterpret_cast<int*>(v[14]);
    TORCH_CHECK(j.p_rows % 32 == 0 && j.p_cols % 4 == 0 && j.p_chunk % 32 == 0 && (v[5] & 15) == 0 &&
                    j.p_inbox_off % 4 == 0 && j.p_inbox_stride % 4 == 0,
                "push job: 32-row groups of 16-byte aligned fp32 rows expected");
  }
  return j;
}

}  // namespace hrm
