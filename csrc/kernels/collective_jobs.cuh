// Fused-collective copy jobs (multi-GPU sharding engine).
//
// Replaces the two FSDP2 collectives of the reference step for the Transformer block weights
// (pretrain.py:119-128, the parameter all-gather; :150-155, the fp32 SUM gradient
// reduce-scatter) with copies over NVLink peer memory that ride inside the GEMM kernels the
// step runs anyway. The epilogue warps of every GEMM CTA run the jobs handed to that launch
// before their first tile (the CTA's TMA and MMA warps start the main loop meanwhile, and the
// first accumulators wait in TMEM), so the transfer overlaps the GEMM's math:
//
//   gather  the bf16 rows of one weight, each from the rank owning it (its shard in the
//           symmetric bf16 buffer), into the local resident copy. Handed to the GEMM that runs
//           just before that weight's first use in the step, so the consuming GEMM reads local
//           memory in its normal tile order and never waits.
//   push    the finished fp32 gradient rows of one weight that other ranks own, into this
//           rank's slot of the owner's inbox, one system-scope count per 32-row x 128-column
//           region on the owner. Handed to the GEMM that runs right after the weight's last
//           gradient contribution of the step. The owners sum the slots and run AdamATan2 at
//           the end of the step (shard_update.cu).
//
// Plain 16-byte loads and stores only (no TMA, no multicast). Neither job waits on anything.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace hrm {

struct CopyJobs {
  // gather (g_src == nullptr: none)
  const unsigned long long* g_src;  // [world] device addresses of each rank's bf16 shard of the weight
  __nv_bfloat16* g_dst;             // local resident copy [g_rows, g_cols]
  int g_rows, g_cols, g_chunk;      // g_chunk: rows per rank shard
  // push (p_src == nullptr: none)
  const float* p_src;               // local fp32 gradient [p_rows, p_cols]
  const unsigned long long* p_base; // [world] fp32 symmetric buffer base addresses
  long p_inbox_off;                 // this weight's shard in inbox slot 0 (fp32 elements from the base)
  long p_inbox_stride;              // fp32 elements between source-rank slots
  long p_cnt_off;                   // this weight's owner-side counts (int32 elements from the base)
  int p_rows, p_cols, p_chunk, p_rank;
  int* p_ran;                       // local flag set to 1 when the push ran (zeroed every step)
};

constexpr int kGatherGranule = 1024;  // bf16 elements (2 KB): four 16-byte loads per lane

// Run by `nw` warps (global warp index `wid`) of a grid; warp-uniform control flow.
__device__ __forceinline__ void run_copy_jobs(const CopyJobs& j, int wid, int nw, int lane) {
  if (j.g_src != nullptr) {
    const long total = (long)j.g_rows * j.g_cols;
    const long chunk_elems = (long)j.g_chunk * j.g_cols;
    const long granules = (total + kGatherGranule - 1) / kGatherGranule;
    for (long g = wid; g < granules; g += nw) {
      const long e0 = g * kGatherGranule;
      uint4 v[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const long e = e0 + (long)(q * 32 + lane) * 8;
        if (e < total) {
          const int owner = (int)((e / j.g_cols) / j.g_chunk);
          v[q] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(j.g_src[owner]) +
                                                      (e - owner * chunk_elems)));
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const long e = e0 + (long)(q * 32 + lane) * 8;
        if (e < total) *reinterpret_cast<uint4*>(j.g_dst + e) = v[q];
      }
    }
  }
  if (j.p_src != nullptr) {
    const int groups = j.p_rows / 32;
    const int cchunks = (j.p_cols + 127) / 128;
    const int total = groups * cchunks;
    for (int g = wid; g < total; g += nw) {
      const int grp = g / cchunks, cc = g % cchunks;
      const int r0 = grp * 32;
      const int owner = r0 / j.p_chunk;
      if (owner == j.p_rank) continue;  // the owner reads its own rows locally
      const int c = cc * 128 + lane * 4;
      float* inbox = reinterpret_cast<float*>(j.p_base[owner]) + j.p_inbox_off + (long)j.p_rank * j.p_inbox_stride +
                     (long)(r0 - owner * j.p_chunk) * j.p_cols;
      if (c < j.p_cols) {
#pragma unroll 1
        for (int rb = 0; rb < 32; rb += 8) {
          float4 v[8];
#pragma unroll
          for (int r = 0; r < 8; ++r)
            v[r] = *reinterpret_cast<const float4*>(j.p_src + (long)(r0 + rb + r) * j.p_cols + c);
#pragma unroll
          for (int r = 0; r < 8; ++r) *reinterpret_cast<float4*>(inbox + (long)(rb + r) * j.p_cols + c) = v[r];
        }
      }
      __threadfence_system();  // the region is visible to the owner before it is counted
      __syncwarp();
      if (lane == 0) {
        int* cnt = reinterpret_cast<int*>(reinterpret_cast<float*>(j.p_base[owner]) + j.p_cnt_off);
        atomicAdd_system(cnt + (r0 - owner * j.p_chunk) / 32, 1);
      }
    }
    if (wid == 0 && lane == 0) *j.p_ran = 1;
  }
}

}  // namespace hrm
