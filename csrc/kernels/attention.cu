// PrefixLM packed-varlen flash attention, forward and backward (head_dim 128, bf16).
//
// Mask (one pass, one LSE): in a document with prefix length P (P = 0 for causal attention),
// query i sees key j iff  j < max(P, i + 1).  Keys never cross documents; tokens after the
// last document (padding) get zero outputs and zero gradients. This is the union of the
// reference's two FlashAttention-3 passes (models/flash_attention_prefixlm_v2.py:88-131:
// bidirectional over the prefix, then bottom-right causal for the response against the
// whole document), computed in a single pass with a single softmax.
//
// Inputs come straight from the fused gqkv projection output [T, 4*H*128] (gate, q, k, v
// heads; q and k already rotated), outputs:
//   forward : O [T, H*128] (ungated), Y = sigmoid(gate) * O [T, H*128], LSE (log2 units) [H, T]
//   backward: d(gate|q|k|v) [T, 4*H*128] with the RoPE backward applied to dq and dk.
//
// Scheduling: attn_schedule builds, on the device, the list of (document, 128-row tile)
// work items ordered longest-first (counting sort by key-block count), so launches have a
// fixed size (CUDA-graph friendly) and persistent CTAs pull items from an atomic counter.
//
// Tensor-core path: warp-level mma.sync m16n8k16 (bf16 -> fp32) with ldmatrix operand loads
// from XOR-swizzled shared memory and cp.async double buffering.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "device_setup.h"

namespace hrm {
namespace attn {

constexpr int D = 128;           // head dim
constexpr int ROW_BYTES = D * 2;  // 256 B per row in shared memory
constexpr int kCostBuckets = 1024;

// ---------------------------------------------------------------------------------------
// small PTX helpers
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(uint32_t smem, const void* gmem, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Byte offset of 16-byte chunk `chunk` of row `row` in a swizzled [rows][128 bf16] tile.
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)(row * ROW_BYTES + ((chunk ^ (row & 7)) << 4));
}

// Load `rows` rows of 128 bf16 starting at token `tok0` (row stride `ld` elements, column
// offset `col`) into a swizzled tile; rows with token >= `tok_end` are zero-filled.
template <int ROWS, int THREADS>
__device__ __forceinline__ void load_tile(uint32_t smem, const __nv_bfloat16* base, long ld, int col, int tok0,
                                          int tok_end) {
#pragma unroll
  for (int i = threadIdx.x; i < ROWS * 16; i += THREADS) {
    const int r = i >> 4, c = i & 15;
    const int tok = tok0 + r;
    const bool valid = tok < tok_end;
    const __nv_bfloat16* src = base + (long)(valid ? tok : 0) * ld + col + c * 8;
    cp_async16(smem + swz(r, c), src, valid);
  }
}

struct Tile {
  int doc_start, len, prefix, pos0;  // pos0: first query (fwd) or first key (bwd) of the tile
};

// ---------------------------------------------------------------------------------------
// schedule
// ---------------------------------------------------------------------------------------
// sched layout (int32): [0] n_fwd, [1] n_bwd, [2] total tokens, [3] n_docs,
// [4..7] work counters (fwd next, fwd done, bwd next, bwd done), then the int4 tile lists.
constexpr int SCHED_HEADER = 8;

__device__ __forceinline__ int fwd_cost(int len, int prefix, int q0) {
  const int kmax = min(len, max(prefix, q0 + 128));
  return (kmax + 63) / 64;
}
__device__ __forceinline__ int bwd_cost(int len, int prefix, int k0) {
  const int qstart = k0 < prefix ? 0 : k0;
  return (len - qstart + 63) / 64;
}

// A packing whose last boundary lies past T, or whose tile lists would overflow `cap`, is
// rejected as a whole: both lists are left empty and the total is set to 0 (so the tail
// kernels zero every output row), and kErrBounds is reported to `err` (if non-null). Nothing
// is then read or written outside the T rows.
__global__ void __launch_bounds__(1024) schedule_kernel(const int* cu, const int* prefix_lens, int n_cu,
                                                        int causal, int cap, int T, int* sched, int* err) {
  __shared__ int hist_f[kCostBuckets], hist_b[kCostBuckets];
  __shared__ int first_bad, tot_f, tot_b, reject;
  int4* fwd_tiles = reinterpret_cast<int4*>(sched + SCHED_HEADER);
  int4* bwd_tiles = fwd_tiles + cap;
  for (int i = threadIdx.x; i < kCostBuckets; i += blockDim.x) hist_f[i] = hist_b[i] = 0;
  if (threadIdx.x == 0) first_bad = n_cu - 1;
  __syncthreads();
  for (int i = threadIdx.x; i < n_cu - 1; i += blockDim.x)
    if (cu[i + 1] <= cu[i]) atomicMin(&first_bad, i);
  __syncthreads();
  const int n_docs = first_bad;

  for (int d = threadIdx.x; d < n_docs; d += blockDim.x) {
    const int len = cu[d + 1] - cu[d];
    const int p = causal ? 0 : min(prefix_lens[d], len);
    for (int q0 = 0; q0 < len; q0 += 128) atomicAdd(&hist_f[min(fwd_cost(len, p, q0), kCostBuckets - 1)], 1);
    for (int k0 = 0; k0 < len; k0 += 128) atomicAdd(&hist_b[min(bwd_cost(len, p, k0), kCostBuckets - 1)], 1);
  }
  __syncthreads();
  // descending-cost exclusive scan (serial over buckets; 1024 adds, negligible)
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int b = kCostBuckets - 1; b >= 0; --b) {
      const int c = hist_f[b];
      hist_f[b] = acc;
      acc += c;
    }
    tot_f = acc;
  } else if (threadIdx.x == 32) {
    int acc = 0;
    for (int b = kCostBuckets - 1; b >= 0; --b) {
      const int c = hist_b[b];
      hist_b[b] = acc;
      acc += c;
    }
    tot_b = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int total = n_docs > 0 ? cu[n_docs] : 0;
    reject = (n_docs > 0 && (cu[0] < 0 || total > T)) || tot_f > cap || tot_b > cap;
    sched[0] = reject ? 0 : tot_f;
    sched[1] = reject ? 0 : tot_b;
    sched[2] = reject ? 0 : total;
    sched[3] = reject ? 0 : n_docs;
    sched[4] = sched[5] = sched[6] = sched[7] = 0;
    if (reject) report_error(err, kErrBounds, 50);
  }
  __syncthreads();
  if (reject) return;
  for (int d = threadIdx.x; d < n_docs; d += blockDim.x) {
    const int start = cu[d];
    const int len = cu[d + 1] - start;
    const int p = causal ? 0 : min(prefix_lens[d], len);
    for (int q0 = 0; q0 < len; q0 += 128) {
      const int slot = atomicAdd(&hist_f[min(fwd_cost(len, p, q0), kCostBuckets - 1)], 1);
      fwd_tiles[slot] = make_int4(start, len, p, q0);
    }
    for (int k0 = 0; k0 < len; k0 += 128) {
      const int slot = atomicAdd(&hist_b[min(bwd_cost(len, p, k0), kCostBuckets - 1)], 1);
      bwd_tiles[slot] = make_int4(start, len, p, k0);
    }
  }
}

// Pull the next work item (persistent CTAs); the last CTA to finish resets the counters so
// the same schedule serves every layer's launch.
__device__ __forceinline__ int next_item(int* counter, int* s_item) {
  __syncthreads();
  if (threadIdx.x == 0) *s_item = atomicAdd(counter, 1);
  __syncthreads();
  return *s_item;
}
__device__ __forceinline__ void finish_cta(int* counter, int* done) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(done, 1) == (int)gridDim.x - 1) {
      *counter = 0;
      *done = 0;
      __threadfence();
    }
  }
}

// ---------------------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------------------
constexpr int FWD_BM = 128, FWD_BN = 64, FWD_THREADS = 256;
constexpr int FWD_SMEM = FWD_BM * ROW_BYTES + 4 * FWD_BN * ROW_BYTES;  // Q + 2x(K,V) = 96 KB

struct FwdParams {
  const __nv_bfloat16* qkv;  // [T, 4*H*D]
  long ld_qkv;
  __nv_bfloat16* out;  // O [T, H*D]
  __nv_bfloat16* y;    // gated [T, H*D]
  long ld_out;
  float* lse;  // [H, T]
  int T, H;
  float scale_log2;
  int* sched;
  int cap;
};

__global__ void __launch_bounds__(FWD_THREADS, 1) attn_fwd_kernel(const FwdParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_item;
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + FWD_BM * ROW_BYTES;
  const uint32_t sV0 = sK0 + 2 * FWD_BN * ROW_BYTES;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int4* tiles = reinterpret_cast<const int4*>(p.sched + SCHED_HEADER);
  const int n_items = p.sched[0] * p.H;

  while (true) {
    const int item = next_item(&p.sched[4], &s_item);
    if (item >= n_items) break;
    const int4 t = tiles[item / p.H];
    const int head = item % p.H;
    const int doc_start = t.x, len = t.y, prefix = t.z, q0 = t.w;
    const int kmax = min(len, max(prefix, q0 + FWD_BM));
    const int n_kb = (kmax + FWD_BN - 1) / FWD_BN;
    const int full_until = min(len, max(prefix, q0 + 1));  // keys < this are visible to every row
    const int q_col = (p.H + head) * D, k_col = (2 * p.H + head) * D, v_col = (3 * p.H + head) * D;
    const int doc_end = doc_start + len;

    load_tile<FWD_BM, FWD_THREADS>(sQ, p.qkv, p.ld_qkv, q_col, doc_start + q0, doc_end);
    load_tile<FWD_BN, FWD_THREADS>(sK0, p.qkv, p.ld_qkv, k_col, doc_start, doc_end);
    load_tile<FWD_BN, FWD_THREADS>(sV0, p.qkv, p.ld_qkv, v_col, doc_start, doc_end);
    cp_async_commit();

    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    const int wrow = warp * 16;  // this warp's first row within the tile
    const int r_lo = lane >> 2, c_lo = (lane & 3) * 2;
    const int qi0 = q0 + wrow + r_lo, qi1 = qi0 + 8;  // doc-relative query indices of this thread
    const int lim0 = max(prefix, qi0 + 1), lim1 = max(prefix, qi1 + 1);

    for (int kb = 0; kb < n_kb; ++kb) {
      const int buf = kb & 1;
      if (kb + 1 < n_kb) {
        const uint32_t nk = sK0 + (buf ^ 1) * FWD_BN * ROW_BYTES, nv = sV0 + (buf ^ 1) * FWD_BN * ROW_BYTES;
        load_tile<FWD_BN, FWD_THREADS>(nk, p.qkv, p.ld_qkv, k_col, doc_start + (kb + 1) * FWD_BN, doc_end);
        load_tile<FWD_BN, FWD_THREADS>(nv, p.qkv, p.ld_qkv, v_col, doc_start + (kb + 1) * FWD_BN, doc_end);
        cp_async_commit();
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();
      const uint32_t sK = sK0 + buf * FWD_BN * ROW_BYTES, sV = sV0 + buf * FWD_BN * ROW_BYTES;

      // S = Q K^T for this warp's 16 rows x 64 keys
      float s[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ks += 2) {
        // Q fragments for k-steps ks, ks+1 (re-read from shared memory: keeps registers free)
        uint32_t qa[4], qb[4];
        {
          const int r = wrow + (lane & 7) + ((lane >> 3) & 1) * 8;
          ldmatrix_x4(sQ + swz(r, ks * 2 + (lane >> 4)), qa[0], qa[1], qa[2], qa[3]);
          ldmatrix_x4(sQ + swz(r, ks * 2 + 2 + (lane >> 4)), qb[0], qb[1], qb[2], qb[3]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(sK + swz(j * 8 + (lane & 7), ks * 2 + (lane >> 3)), b0, b1, b2, b3);
          mma_bf16(s[j], qa[0], qa[1], qa[2], qa[3], b0, b1);
          mma_bf16(s[j], qb[0], qb[1], qb[2], qb[3], b2, b3);
        }
      }
      // scale (log2 domain) + mask
      const int k_base = kb * FWD_BN;
      const bool need_mask = k_base + FWD_BN > full_until;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float v = s[j][e] * p.scale_log2;
          if (need_mask) {
            const int key = k_base + j * 8 + c_lo + (e & 1);
            const int lim = (e < 2) ? lim0 : lim1;
            if (key >= len || key >= lim) v = -INFINITY;
          }
          s[j][e] = v;
        }
      }
      // online softmax per row (two rows per thread: r_lo and r_lo + 8)
      float mx[2] = {m_run[0], m_run[1]};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        mx[0] = fmaxf(mx[0], fmaxf(s[j][0], s[j][1]));
        mx[1] = fmaxf(mx[1], fmaxf(s[j][2], s[j][3]));
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffff, mx[h], 1));
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffff, mx[h], 2));
      }
      float alpha[2], rs[2] = {0.f, 0.f};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float safe = mx[h] == -INFINITY ? 0.f : mx[h];
        alpha[h] = fast_exp2(m_run[h] - safe);
        m_run[h] = mx[h];
        mx[h] = safe;
      }
      uint32_t pf[8][2];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float p0 = fast_exp2(s[j][0] - mx[0]), p1 = fast_exp2(s[j][1] - mx[0]);
        const float p2 = fast_exp2(s[j][2] - mx[1]), p3 = fast_exp2(s[j][3] - mx[1]);
        rs[0] += p0 + p1;
        rs[1] += p2 + p3;
        pf[j][0] = pack_bf16x2(p0, p1);
        pf[j][1] = pack_bf16x2(p2, p3);
      }
      l_run[0] = l_run[0] * alpha[0] + rs[0];
      l_run[1] = l_run[1] * alpha[1] + rs[1];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][0] *= alpha[0];
        o[j][1] *= alpha[0];
        o[j][2] *= alpha[1];
        o[j][3] *= alpha[1];
      }
      // O += P V : k = 64 keys (4 steps of 16), n = 128 dims (16 tiles of 8)
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t a0 = pf[2 * kk][0], a1 = pf[2 * kk][1], a2 = pf[2 * kk + 1][0], a3 = pf[2 * kk + 1][1];
#pragma unroll
        for (int jn = 0; jn < 16; jn += 2) {
          uint32_t b0, b1, b2, b3;
          const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = jn + (lane >> 4);
          ldmatrix_x4_trans(sV + swz(r, c), b0, b1, b2, b3);
          mma_bf16(o[jn], a0, a1, a2, a3, b0, b1);
          mma_bf16(o[jn + 1], a0, a1, a2, a3, b2, b3);
        }
      }
      __syncthreads();
    }

    // finalise: row sums across the quad, normalise, stage in shared memory (own rows of sQ)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      l_run[h] += __shfl_xor_sync(0xffffffff, l_run[h], 1);
      l_run[h] += __shfl_xor_sync(0xffffffff, l_run[h], 2);
    }
    const float inv0 = l_run[0] > 0.f ? 1.f / l_run[0] : 0.f;
    const float inv1 = l_run[1] > 0.f ? 1.f / l_run[1] : 0.f;
    uint8_t* sQb = smem;
#pragma unroll
    for (int j = 0; j < 16; ++j) {  // n-tile j = 16-byte chunk j; this thread owns columns j*8 + c_lo, +1
      const int r0 = wrow + r_lo, r1 = r0 + 8;
      *reinterpret_cast<uint32_t*>(sQb + swz(r0, j) + c_lo * 2) = pack_bf16x2(o[j][0] * inv0, o[j][1] * inv0);
      *reinterpret_cast<uint32_t*>(sQb + swz(r1, j) + c_lo * 2) = pack_bf16x2(o[j][2] * inv1, o[j][3] * inv1);
    }
    if ((lane & 3) == 0) {
      const int t0 = doc_start + qi0, t1 = doc_start + qi1;
      if (qi0 < len) p.lse[(long)head * p.T + t0] = m_run[0] + __log2f(l_run[0]);
      if (qi1 < len) p.lse[(long)head * p.T + t1] = m_run[1] + __log2f(l_run[1]);
    }
    __syncwarp();
    // coalesced write of O and the gated output Y = sigmoid(gate) * O for this warp's rows
#pragma unroll
    for (int i = lane; i < 16 * 16; i += 32) {
      const int r = wrow + (i >> 4), c = i & 15;
      const int qi = q0 + r;
      if (qi < len) {
        const long tok = doc_start + qi;
        const uint4 ov = *reinterpret_cast<const uint4*>(sQb + swz(r, c));
        const uint4 gv = *reinterpret_cast<const uint4*>(p.qkv + tok * p.ld_qkv + head * D + c * 8);
        uint4 yv;
        const uint32_t* oa = &ov.x;
        const uint32_t* ga = &gv.x;
        uint32_t* ya = &yv.x;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const float2 of = unpack_bf16x2(oa[w]), gf = unpack_bf16x2(ga[w]);
          ya[w] = pack_bf16x2(of.x * sigmoidf_(gf.x), of.y * sigmoidf_(gf.y));
        }
        *reinterpret_cast<uint4*>(p.out + tok * p.ld_out + head * D + c * 8) = ov;
        *reinterpret_cast<uint4*>(p.y + tok * p.ld_out + head * D + c * 8) = yv;
      }
    }
  }
  finish_cta(&p.sched[4], &p.sched[5]);
}

// Zero O, Y and LSE for padding tokens [total, T).
__global__ void attn_zero_tail_kernel(__nv_bfloat16* out, __nv_bfloat16* y, long ld_out, float* lse, int T, int H,
                                      const int* sched) {
  const int total = sched[2];
  const int width = H * D;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < (long)(T - total) * (width / 8);
       i += (long)gridDim.x * blockDim.x) {
    const long tok = total + i / (width / 8);
    const int c = (int)(i % (width / 8)) * 8;
    *reinterpret_cast<uint4*>(out + tok * ld_out + c) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(y + tok * ld_out + c) = make_uint4(0, 0, 0, 0);
  }
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < (long)(T - total) * H;
       i += (long)gridDim.x * blockDim.x) {
    const int h = (int)(i % H);
    const long tok = total + i / H;
    lse[(long)h * T + tok] = 0.f;
  }
}

// ---------------------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------------------
// Preprocess: dO = dY * sigmoid(g); d(gate) = dY * O * s * (1 - s); Dsum = rowsum(dO * O);
// zero the fp32 dQ accumulator. One warp per (token, head); 4 dims per lane.
__global__ void attn_bwd_pre_kernel(const __nv_bfloat16* dy, const __nv_bfloat16* out, long ld_out,
                                    const __nv_bfloat16* qkv, long ld_qkv, __nv_bfloat16* d_out,
                                    __nv_bfloat16* dqkv, long ld_dqkv, float* dsum, float* dq_acc, int T, int H) {
  const long gw = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= (long)T * H) return;
  const long tok = gw / H;
  const int head = (int)(gw % H);
  const long o_off = tok * ld_out + head * D + lane * 4;
  const uint2 dyv = *reinterpret_cast<const uint2*>(dy + o_off);
  const uint2 ov = *reinterpret_cast<const uint2*>(out + o_off);
  const uint2 gv = *reinterpret_cast<const uint2*>(qkv + tok * ld_qkv + head * D + lane * 4);
  const float2 dy0 = unpack_bf16x2(dyv.x), dy1 = unpack_bf16x2(dyv.y);
  const float2 o0 = unpack_bf16x2(ov.x), o1 = unpack_bf16x2(ov.y);
  const float2 g0 = unpack_bf16x2(gv.x), g1 = unpack_bf16x2(gv.y);
  const float dyf[4] = {dy0.x, dy0.y, dy1.x, dy1.y}, of[4] = {o0.x, o0.y, o1.x, o1.y},
              gf[4] = {g0.x, g0.y, g1.x, g1.y};
  float dof[4], dgf[4], acc = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float sg = sigmoidf_(gf[i]);
    dof[i] = bf16_round(dyf[i] * sg);
    dgf[i] = dyf[i] * of[i] * sg * (1.f - sg);
    acc += dof[i] * of[i];
  }
  *reinterpret_cast<uint2*>(d_out + o_off) = make_uint2(pack_bf16x2(dof[0], dof[1]), pack_bf16x2(dof[2], dof[3]));
  *reinterpret_cast<uint2*>(dqkv + tok * ld_dqkv + head * D + lane * 4) =
      make_uint2(pack_bf16x2(dgf[0], dgf[1]), pack_bf16x2(dgf[2], dgf[3]));
  *reinterpret_cast<float4*>(dq_acc + tok * (long)(H * D) + head * D + lane * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffff, acc, off);
  if (lane == 0) dsum[(long)head * T + tok] = acc;
}

constexpr int BWD_BN = 128, BWD_BM = 64, BWD_THREADS = 256;
// K, V (128 rows each), Q and dO double-buffered (64 rows each), dS [64 q][128 keys]
constexpr int BWD_SMEM = 2 * BWD_BN * ROW_BYTES + 4 * BWD_BM * ROW_BYTES + BWD_BM * ROW_BYTES + 4 * BWD_BM * 4;

struct BwdParams {
  const __nv_bfloat16* qkv;
  long ld_qkv;
  const __nv_bfloat16* d_out;  // dO [T, H*D]
  long ld_out;
  const float* lse;   // [H, T]
  const float* dsum;  // [H, T]
  float* dq_acc;      // [T, H*D] fp32
  __nv_bfloat16* dqkv;
  long ld_dqkv;
  const int* positions;
  const float* cos_tab;  // [S, 64]
  const float* sin_tab;
  int T, H;
  float scale;       // softmax scale (natural units)
  float scale_log2;  // scale * log2(e)
  int* sched;
  int cap;
};

__global__ void __launch_bounds__(BWD_THREADS, 1) attn_bwd_kernel(const BwdParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_item;
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + BWD_BN * ROW_BYTES;
  const uint32_t sQ0 = sV + BWD_BN * ROW_BYTES;             // 2 buffers of 64 rows
  const uint32_t sO0 = sQ0 + 2 * BWD_BM * ROW_BYTES;        // dO, 2 buffers
  const uint32_t sS = sO0 + 2 * BWD_BM * ROW_BYTES;         // dS [64][128] bf16 (swizzled rows of 256 B)
  float* sL = reinterpret_cast<float*>(smem + (sS - sK) + BWD_BM * ROW_BYTES);  // lse [2][64]
  float* sDs = sL + 2 * BWD_BM;                                                  // dsum [2][64]
  uint8_t* sSb = smem + (sS - sK);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r_lo = lane >> 2, c_lo = (lane & 3) * 2;
  const int4* tiles = reinterpret_cast<const int4*>(p.sched + SCHED_HEADER) + p.cap;
  const int n_items = p.sched[1] * p.H;

  while (true) {
    const int item = next_item(&p.sched[6], &s_item);
    if (item >= n_items) break;
    const int4 t = tiles[item / p.H];
    const int head = item % p.H;
    const int doc_start = t.x, len = t.y, prefix = t.z, k0 = t.w;
    const int doc_end = doc_start + len;
    const int qstart = k0 < prefix ? 0 : k0;
    const int n_qb = (len - qstart + BWD_BM - 1) / BWD_BM;
    const int q_col = (p.H + head) * D, k_col = (2 * p.H + head) * D, v_col = (3 * p.H + head) * D;

    load_tile<BWD_BN, BWD_THREADS>(sK, p.qkv, p.ld_qkv, k_col, doc_start + k0, doc_end);
    load_tile<BWD_BN, BWD_THREADS>(sV, p.qkv, p.ld_qkv, v_col, doc_start + k0, doc_end);
    auto load_q_block = [&](int qb, int buf) {
      const int q_tok = doc_start + qstart + qb * BWD_BM;
      load_tile<BWD_BM, BWD_THREADS>(sQ0 + buf * BWD_BM * ROW_BYTES, p.qkv, p.ld_qkv, q_col, q_tok, doc_end);
      load_tile<BWD_BM, BWD_THREADS>(sO0 + buf * BWD_BM * ROW_BYTES, p.d_out, p.ld_out, head * D, q_tok, doc_end);
      if (threadIdx.x < BWD_BM) {
        const int tok = q_tok + threadIdx.x;
        const bool ok = tok < doc_end;
        sL[buf * BWD_BM + threadIdx.x] = ok ? p.lse[(long)head * p.T + tok] : 0.f;
        sDs[buf * BWD_BM + threadIdx.x] = ok ? p.dsum[(long)head * p.T + tok] : 0.f;
      }
    };
    load_q_block(0, 0);
    cp_async_commit();

    float dk[16][4], dv[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) dk[j][e] = dv[j][e] = 0.f;

    const int wkey = warp * 16;  // this warp's keys within the block
    const int key0 = k0 + wkey + r_lo, key1 = key0 + 8;  // doc-relative keys of this thread's rows

    for (int qb = 0; qb < n_qb; ++qb) {
      const int buf = qb & 1;
      if (qb + 1 < n_qb) {
        load_q_block(qb + 1, buf ^ 1);
        cp_async_commit();
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();
      const uint32_t sQ = sQ0 + buf * BWD_BM * ROW_BYTES, sO = sO0 + buf * BWD_BM * ROW_BYTES;
      const float* lseb = sL + buf * BWD_BM;
      const float* dsb = sDs + buf * BWD_BM;
      const int qbase = qstart + qb * BWD_BM;  // doc-relative first query of the block

      // S^T = K_w Q^T and dP^T = V_w dO^T : 16 keys x 64 queries per warp
      float st[8][4], dpt[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) st[j][e] = dpt[j][e] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t ka0, ka1, ka2, ka3, va0, va1, va2, va3;
        const int ar = wkey + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int ac = ks * 2 + (lane >> 4);
        ldmatrix_x4(sK + swz(ar, ac), ka0, ka1, ka2, ka3);
        ldmatrix_x4(sV + swz(ar, ac), va0, va1, va2, va3);
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
          uint32_t q0_, q1_, q2_, q3_, o0_, o1_, o2_, o3_;
          // rows j*8..j*8+15 (queries), k chunk ks*2 (+1): x4 covers two n-tiles
          const int br = j * 8 + (lane & 7) + ((lane >> 4) & 1) * 8;
          const int bc = ks * 2 + ((lane >> 3) & 1);
          ldmatrix_x4(sQ + swz(br, bc), q0_, q1_, q2_, q3_);
          ldmatrix_x4(sO + swz(br, bc), o0_, o1_, o2_, o3_);
          mma_bf16(st[j], ka0, ka1, ka2, ka3, q0_, q1_);
          mma_bf16(st[j + 1], ka0, ka1, ka2, ka3, q2_, q3_);
          mma_bf16(dpt[j], va0, va1, va2, va3, o0_, o1_);
          mma_bf16(dpt[j + 1], va0, va1, va2, va3, o2_, o3_);
        }
      }
      // P^T, dS^T (registers). Element (key row, query col).
      uint32_t pt[8][2], dst[8][2];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float pv[4], dsv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int qcol = j * 8 + c_lo + (e & 1);
          const int q = qbase + qcol;
          const int key = (e < 2) ? key0 : key1;
          const bool vis = q < len && key < len && key < max(prefix, q + 1);
          const float pr = vis ? fast_exp2(st[j][e] * p.scale_log2 - lseb[qcol]) : 0.f;
          pv[e] = pr;
          dsv[e] = pr * (dpt[j][e] - dsb[qcol]) * p.scale;
        }
        pt[j][0] = pack_bf16x2(pv[0], pv[1]);
        pt[j][1] = pack_bf16x2(pv[2], pv[3]);
        dst[j][0] = pack_bf16x2(dsv[0], dsv[1]);
        dst[j][1] = pack_bf16x2(dsv[2], dsv[3]);
        // stash dS (transposed: row = query, col = key) for the dQ product
        const int kcol = wkey + r_lo;
        uint16_t* row0 = reinterpret_cast<uint16_t*>(sSb + swz(j * 8 + c_lo, kcol >> 3)) + (kcol & 7);
        uint16_t* row1 = reinterpret_cast<uint16_t*>(sSb + swz(j * 8 + c_lo + 1, kcol >> 3)) + (kcol & 7);
        uint16_t* row2 = reinterpret_cast<uint16_t*>(sSb + swz(j * 8 + c_lo, (kcol + 8) >> 3)) + ((kcol + 8) & 7);
        uint16_t* row3 = reinterpret_cast<uint16_t*>(sSb + swz(j * 8 + c_lo + 1, (kcol + 8) >> 3)) + ((kcol + 8) & 7);
        *row0 = (uint16_t)(dst[j][0] & 0xffff);
        *row1 = (uint16_t)(dst[j][0] >> 16);
        *row2 = (uint16_t)(dst[j][1] & 0xffff);
        *row3 = (uint16_t)(dst[j][1] >> 16);
      }
      // dV += P^T dO ; dK += dS^T Q  (k = 64 queries in 4 steps, n = 128 dims)
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t pa0 = pt[2 * kk][0], pa1 = pt[2 * kk][1], pa2 = pt[2 * kk + 1][0], pa3 = pt[2 * kk + 1][1];
        const uint32_t da0 = dst[2 * kk][0], da1 = dst[2 * kk][1], da2 = dst[2 * kk + 1][0],
                       da3 = dst[2 * kk + 1][1];
#pragma unroll
        for (int jn = 0; jn < 16; jn += 2) {
          uint32_t b0, b1, b2, b3;
          const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = jn + (lane >> 4);
          ldmatrix_x4_trans(sO + swz(r, c), b0, b1, b2, b3);
          mma_bf16(dv[jn], pa0, pa1, pa2, pa3, b0, b1);
          mma_bf16(dv[jn + 1], pa0, pa1, pa2, pa3, b2, b3);
          ldmatrix_x4_trans(sQ + swz(r, c), b0, b1, b2, b3);
          mma_bf16(dk[jn], da0, da1, da2, da3, b0, b1);
          mma_bf16(dk[jn + 1], da0, da1, da2, da3, b2, b3);
        }
      }
      __syncthreads();  // dS complete in shared memory
      // dQ (64 x 128) += dS (64 x 128 keys) K (128 keys x 128 dims); warp -> 16 rows x 64 dims
      {
        const int wq = (warp & 3) * 16, wd = (warp >> 2) * 64;
        float dq[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) dq[j][0] = dq[j][1] = dq[j][2] = dq[j][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          uint32_t a0, a1, a2, a3;
          const int ar = wq + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int ac = ks * 2 + (lane >> 4);
          ldmatrix_x4(sS + swz(ar, ac), a0, a1, a2, a3);
#pragma unroll
          for (int jn = 0; jn < 8; jn += 2) {
            uint32_t b0, b1, b2, b3;
            const int r = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
            const int c = (wd >> 3) + jn + (lane >> 4);
            ldmatrix_x4_trans(sK + swz(r, c), b0, b1, b2, b3);
            mma_bf16(dq[jn], a0, a1, a2, a3, b0, b1);
            mma_bf16(dq[jn + 1], a0, a1, a2, a3, b2, b3);
          }
        }
        const int q_r0 = qbase + wq + r_lo, q_r1 = q_r0 + 8;
#pragma unroll
        for (int jn = 0; jn < 8; jn += 2) {
          // pairs of n-tiles give 4 consecutive... use float2 atomics per n-tile
          const int col = head * D + wd + jn * 8 + c_lo;
          if (q_r0 < len) {
            float* dst0 = p.dq_acc + (long)(doc_start + q_r0) * (p.H * D) + col;
            atomicAdd(reinterpret_cast<float2*>(dst0), make_float2(dq[jn][0], dq[jn][1]));
            atomicAdd(reinterpret_cast<float2*>(dst0 + 8), make_float2(dq[jn + 1][0], dq[jn + 1][1]));
          }
          if (q_r1 < len) {
            float* dst1 = p.dq_acc + (long)(doc_start + q_r1) * (p.H * D) + col;
            atomicAdd(reinterpret_cast<float2*>(dst1), make_float2(dq[jn][2], dq[jn][3]));
            atomicAdd(reinterpret_cast<float2*>(dst1 + 8), make_float2(dq[jn + 1][2], dq[jn + 1][3]));
          }
        }
      }
      __syncthreads();  // before the next block overwrites dS / buffers
    }

    // dK: apply the RoPE backward (pairs d, d+64 live in n-tiles j, j+8 of this thread),
    // then write dK and dV rows of this warp's keys.
    const float* cos_t = p.cos_tab;
    const float* sin_t = p.sin_tab;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int key = half ? key1 : key0;
      if (key < len) {
        const long tok = doc_start + key;
        const int pos = p.positions[tok];
        __nv_bfloat16* dk_row = p.dqkv + tok * p.ld_dqkv + (2 * p.H + head) * D;
        __nv_bfloat16* dv_row = p.dqkv + tok * p.ld_dqkv + (3 * p.H + head) * D;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int d = j * 8 + c_lo;
          const float c0 = cos_t[pos * 64 + d], c1 = cos_t[pos * 64 + d + 1];
          const float s0 = sin_t[pos * 64 + d], s1 = sin_t[pos * 64 + d + 1];
          const float x1a = dk[j][half * 2], x1b = dk[j][half * 2 + 1];
          const float x2a = dk[j + 8][half * 2], x2b = dk[j + 8][half * 2 + 1];
          *reinterpret_cast<uint32_t*>(dk_row + d) = pack_bf16x2(x1a * c0 + x2a * s0, x1b * c1 + x2b * s1);
          *reinterpret_cast<uint32_t*>(dk_row + d + 64) = pack_bf16x2(x2a * c0 - x1a * s0, x2b * c1 - x1b * s1);
          *reinterpret_cast<uint32_t*>(dv_row + d) = pack_bf16x2(dv[j][half * 2], dv[j][half * 2 + 1]);
          *reinterpret_cast<uint32_t*>(dv_row + d + 64) = pack_bf16x2(dv[j + 8][half * 2], dv[j + 8][half * 2 + 1]);
        }
      }
    }
  }
  finish_cta(&p.sched[6], &p.sched[7]);
}

// dq = RoPE^T(dq_acc) -> d(q) slice; zero dq/dk/dv slices of padding tokens.
__global__ void attn_bwd_post_kernel(const float* dq_acc, __nv_bfloat16* dqkv, long ld_dqkv, const int* positions,
                                     const float* cos_tab, const float* sin_tab, int rope_rows, int* err, int T, int H,
                                     const int* sched) {
  // 16 threads per (token, head) row, 4 rotation pairs (d, d + 64) each: 16-byte fp32 loads,
  // 8-byte bf16 stores, no 64-bit division per element
  const int total = sched[2];
  const int rows = T * H;
  const int d = (threadIdx.x & 15) * 4;
  const int stride = (int)((gridDim.x * blockDim.x) >> 4);
  for (int r = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 4); r < rows; r += stride) {
    const int tok = r / H, head = r - tok * H;
    __nv_bfloat16* q_row = dqkv + (long)tok * ld_dqkv + (H + head) * D;
    if (tok >= total) {  // padding tokens: zero dQ, dK, dV
      const uint2 z = make_uint2(0u, 0u);
      __nv_bfloat16* k_row = dqkv + (long)tok * ld_dqkv + (2 * H + head) * D;
      __nv_bfloat16* v_row = dqkv + (long)tok * ld_dqkv + (3 * H + head) * D;
      *reinterpret_cast<uint2*>(q_row + d) = z;
      *reinterpret_cast<uint2*>(q_row + d + 64) = z;
      *reinterpret_cast<uint2*>(k_row + d) = z;
      *reinterpret_cast<uint2*>(k_row + d + 64) = z;
      *reinterpret_cast<uint2*>(v_row + d) = z;
      *reinterpret_cast<uint2*>(v_row + d + 64) = z;
      continue;
    }
    const float* src = dq_acc + (long)tok * (H * D) + head * D;
    const float4 a = *reinterpret_cast<const float4*>(src + d);
    const float4 b = *reinterpret_cast<const float4*>(src + d + 64);
    int pos = positions[tok];
    if (!HRM_BOUNDS_OK(pos >= 0 && pos < rope_rows, err, 104)) pos = 0;
    const float4 c = *reinterpret_cast<const float4*>(cos_tab + (long)pos * 64 + d);
    const float4 sn = *reinterpret_cast<const float4*>(sin_tab + (long)pos * 64 + d);
    *reinterpret_cast<uint2*>(q_row + d) = make_uint2(pack_bf16x2(a.x * c.x + b.x * sn.x, a.y * c.y + b.y * sn.y),
                                                      pack_bf16x2(a.z * c.z + b.z * sn.z, a.w * c.w + b.w * sn.w));
    *reinterpret_cast<uint2*>(q_row + d + 64) = make_uint2(pack_bf16x2(b.x * c.x - a.x * sn.x, b.y * c.y - a.y * sn.y),
                                                           pack_bf16x2(b.z * c.z - a.z * sn.z, b.w * c.w - a.w * sn.w));
  }
}

}  // namespace attn

// ---------------------------------------------------------------------------------------
// host API
// ---------------------------------------------------------------------------------------
at::Tensor device_error_word();

int64_t attn_schedule_capacity(int64_t T, int64_t n_cu) { return (T + 127) / 128 + n_cu; }

void attn_schedule(const at::Tensor& cu_seqlens, const at::Tensor& prefix_lens, bool causal, int64_t T,
                   const at::Tensor& sched) {
  TORCH_CHECK(cu_seqlens.scalar_type() == at::kInt && prefix_lens.scalar_type() == at::kInt, "int32 metadata");
  c10::cuda::CUDAGuard guard(cu_seqlens.device());
  const int n_cu = (int)cu_seqlens.numel();
  const int64_t cap = (sched.numel() - attn::SCHED_HEADER) / 8;
  TORCH_CHECK(cap > 0, "schedule buffer too small");
  attn::schedule_kernel<<<1, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(
      cu_seqlens.data_ptr<int>(), prefix_lens.data_ptr<int>(), n_cu, causal ? 1 : 0, (int)cap, (int)T,
      sched.data_ptr<int>(), device_error_word().data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static int sm_count() { return device_sm_count(); }

void attn_fwd(const at::Tensor& qkv, int64_t H, const at::Tensor& sched, const at::Tensor& out, const at::Tensor& y,
              const at::Tensor& lse) {
  c10::cuda::CUDAGuard guard(qkv.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  attn::FwdParams p{};
  p.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  p.ld_qkv = qkv.stride(0);
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.y = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  TORCH_CHECK(out.stride(0) == y.stride(0), "O and Y must share a row stride");
  p.ld_out = out.stride(0);
  p.lse = lse.data_ptr<float>();
  p.T = (int)qkv.size(0);
  p.H = (int)H;
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)attn::D));
  p.sched = sched.data_ptr<int>();
  p.cap = (int)((sched.numel() - attn::SCHED_HEADER) / 8);
  TORCH_CHECK(qkv.size(1) >= 4 * H * attn::D, "qkv width");
  TORCH_CHECK(ensure_dynamic_smem((const void*)attn::attn_fwd_kernel, attn::FWD_SMEM) == cudaSuccess,
              "cudaFuncSetAttribute failed");
  attn::attn_fwd_kernel<<<sm_count(), attn::FWD_THREADS, attn::FWD_SMEM, stream>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  attn::attn_zero_tail_kernel<<<64, 256, 0, stream>>>(p.out, p.y, p.ld_out, p.lse, p.T, p.H, p.sched);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void attn_bwd(const at::Tensor& qkv, int64_t H, const at::Tensor& sched, const at::Tensor& out,
              const at::Tensor& lse, const at::Tensor& dy, const at::Tensor& positions, const at::Tensor& cos_tab,
              const at::Tensor& sin_tab, const at::Tensor& d_out, const at::Tensor& dsum, const at::Tensor& dq_acc,
              const at::Tensor& dqkv) {
  c10::cuda::CUDAGuard guard(qkv.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int T = (int)qkv.size(0);
  {
    const long warps = (long)T * H;
    const int threads = 256;
    const long blocks = (warps * 32 + threads - 1) / threads;
    attn::attn_bwd_pre_kernel<<<(unsigned)blocks, threads, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()),
        out.stride(0), reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0),
        reinterpret_cast<__nv_bfloat16*>(d_out.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()),
        dqkv.stride(0), dsum.data_ptr<float>(), dq_acc.data_ptr<float>(), T, (int)H);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  attn::BwdParams p{};
  p.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  p.ld_qkv = qkv.stride(0);
  p.d_out = reinterpret_cast<const __nv_bfloat16*>(d_out.data_ptr());
  p.ld_out = d_out.stride(0);
  p.lse = lse.data_ptr<float>();
  p.dsum = dsum.data_ptr<float>();
  p.dq_acc = dq_acc.data_ptr<float>();
  p.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  p.ld_dqkv = dqkv.stride(0);
  p.positions = positions.data_ptr<int>();
  p.cos_tab = cos_tab.data_ptr<float>();
  p.sin_tab = sin_tab.data_ptr<float>();
  p.T = T;
  p.H = (int)H;
  p.scale = (float)(1.0 / std::sqrt((double)attn::D));
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)attn::D));
  p.sched = sched.data_ptr<int>();
  p.cap = (int)((sched.numel() - attn::SCHED_HEADER) / 8);
  TORCH_CHECK(ensure_dynamic_smem((const void*)attn::attn_bwd_kernel, attn::BWD_SMEM) == cudaSuccess,
              "cudaFuncSetAttribute failed");
  attn::attn_bwd_kernel<<<sm_count(), attn::BWD_THREADS, attn::BWD_SMEM, stream>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  attn::attn_bwd_post_kernel<<<1024, 256, 0, stream>>>(p.dq_acc, p.dqkv, p.ld_dqkv, p.positions, p.cos_tab,
                                                        p.sin_tab, (int)cos_tab.size(0),
                                                        device_error_word().data_ptr<int>(), T, (int)H, p.sched);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace hrm
