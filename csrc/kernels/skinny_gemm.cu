// Small-M linear layer for the decode step: y[M, *] = x[M, K] * W[*, K]^T for M <= 32 rows
// (one row per sequence being decoded), with the training GEMM's epilogues fused.
//
// At M <= 32 a linear layer is bound by reading W once from HBM; the 128/256-row tensor-core
// tiles of the tcgen05 GEMM (gemm_tcgen05.cu) would leave most of each tile empty and give
// only N / 256 CTAs. Here every warp owns one *pair* of output features and all M rows:
//   EPI_STORE / EPI_RESIDUAL  features (2p, 2p + 1), plus an optional bf16 residual
//   EPI_ROPE                  features (128h + i, 128h + i + 64): the rotate-half partners of
//                             head h, so RoPE (at positions[m]) is applied in registers to
//                             the q / k heads in [rope_begin, rope_end)
//   EPI_SWIGLU                gate row p and up row p + pair_offset -> h = silu(g) * u
// A CTA (8 warps) stages x in shared memory 1024 columns at a time; each lane covers 8
// consecutive k of every 256-wide step with one 16-byte load per weight row, accumulates the
// M x 2 dot products in fp32 registers, and the warp reduces them with shuffles. Values are
// rounded to bf16 before the epilogue math, as the reference rounds the projection output.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "device_setup.h"

namespace hrm {
namespace {

constexpr int SK_WARPS = 8;
constexpr int SK_MAXM = 32;
constexpr int SK_KCHUNK = 1024;
constexpr int SK_SMEM = SK_MAXM * SK_KCHUNK * 2;  // 64 KB of x per chunk

enum SkinnyEpi : int { SK_STORE = 0, SK_RESIDUAL = 1, SK_ROPE = 3, SK_SWIGLU = 4 };

__device__ __forceinline__ void unpack8(const uint4 v, float (&f)[8]) {
  const float2 a = unpack_bf16x2(v.x), b = unpack_bf16x2(v.y), c = unpack_bf16x2(v.z), d = unpack_bf16x2(v.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

struct SkinnyArgs {
  const __nv_bfloat16* x;
  long ldx;
  const __nv_bfloat16* w;
  long ldw;
  int M, K, pairs;
  __nv_bfloat16* out;
  long ldo;
  const __nv_bfloat16* residual;
  long ldr;
  const int* positions;
  const float* cos_tab;  // [max_pos, 64]
  const float* sin_tab;
  int rope_begin, rope_end, pair_offset;
};

template <int EPI>
__global__ void __launch_bounds__(SK_WARPS * 32) skinny_linear_kernel(const SkinnyArgs a) {
  extern __shared__ uint4 sx[];  // [M][SK_KCHUNK / 8] 16-byte chunks
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pair = blockIdx.x * SK_WARPS + warp;
  const bool active = pair < a.pairs;
  int f0 = 0, f1 = 0;  // weight rows of this warp's pair
  if (EPI == SK_ROPE) {
    f0 = (pair >> 6) * 128 + (pair & 63);
    f1 = f0 + 64;
  } else if (EPI == SK_SWIGLU) {
    f0 = pair;
    f1 = pair + a.pair_offset;
  } else {
    f0 = 2 * pair;
    f1 = 2 * pair + 1;
  }
  float acc0[SK_MAXM], acc1[SK_MAXM];
#pragma unroll
  for (int m = 0; m < SK_MAXM; ++m) acc0[m] = acc1[m] = 0.f;
  const int chunks_per_row = SK_KCHUNK / 8;
  for (int k0 = 0; k0 < a.K; k0 += SK_KCHUNK) {
    const int kc = min(SK_KCHUNK, a.K - k0);
    __syncthreads();
    for (int i = threadIdx.x; i < a.M * (kc / 8); i += blockDim.x) {
      const int m = i / (kc / 8), c = i % (kc / 8);
      sx[m * chunks_per_row + c] = *reinterpret_cast<const uint4*>(a.x + (long)m * a.ldx + k0 + c * 8);
    }
    __syncthreads();
    if (active) {
      for (int c = lane; c < kc / 8; c += 32) {
        float w0[8], w1[8];
        unpack8(__ldg(reinterpret_cast<const uint4*>(a.w + (long)f0 * a.ldw + k0 + c * 8)), w0);
        unpack8(__ldg(reinterpret_cast<const uint4*>(a.w + (long)f1 * a.ldw + k0 + c * 8)), w1);
#pragma unroll
        for (int m = 0; m < SK_MAXM; ++m) {
          if (m < a.M) {
            float xv[8];
            unpack8(sx[m * chunks_per_row + c], xv);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              acc0[m] = fmaf(w0[e], xv[e], acc0[m]);
              acc1[m] = fmaf(w1[e], xv[e], acc1[m]);
            }
          }
        }
      }
    }
  }
  if (!active) return;
  // butterfly reduction: afterwards every lane holds the full sums; lane m keeps row m
  float v0 = 0.f, v1 = 0.f;
#pragma unroll
  for (int m = 0; m < SK_MAXM; ++m) {
    float s0 = acc0[m], s1 = acc1[m];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, off);
      s1 += __shfl_xor_sync(0xffffffffu, s1, off);
    }
    if (lane == m) {
      v0 = s0;
      v1 = s1;
    }
  }
  const int m = lane;
  if (m >= a.M) return;
  v0 = bf16_round(v0);
  v1 = bf16_round(v1);
  __nv_bfloat16* orow = a.out + (long)m * a.ldo;
  if constexpr (EPI == SK_SWIGLU) {
    const float h = __fdividef(v0, 1.0f + __expf(-v0)) * v1;  // fast divide: the output is bf16
    orow[pair] = __float2bfloat16_rn(h);
  } else if constexpr (EPI == SK_ROPE) {
    if (f0 >= a.rope_begin && f0 < a.rope_end) {
      const int i = f0 & 63;
      const long pos = a.positions[m];
      const float c = a.cos_tab[pos * 64 + i], s = a.sin_tab[pos * 64 + i];
      const float r0 = v0 * c - v1 * s, r1 = v1 * c + v0 * s;
      v0 = r0;
      v1 = r1;
    }
    orow[f0] = __float2bfloat16_rn(v0);
    orow[f1] = __float2bfloat16_rn(v1);
  } else {
    if constexpr (EPI == SK_RESIDUAL) {
      const float2 r = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(a.residual + (long)m * a.ldr + f0));
      v0 += r.x;
      v1 += r.y;
    }
    *reinterpret_cast<uint32_t*>(orow + f0) = pack_bf16x2(v0, v1);
  }
}

template <int EPI>
void launch_skinny(const SkinnyArgs& a, cudaStream_t stream) {
  auto kern = skinny_linear_kernel<EPI>;
  TORCH_CHECK(ensure_dynamic_smem((const void*)kern, SK_SMEM) == cudaSuccess, "cudaFuncSetAttribute failed");
  const int grid = (a.pairs + SK_WARPS - 1) / SK_WARPS;
  kern<<<grid, SK_WARPS * 32, SK_SMEM, stream>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace

// x [M <= 32, K] bf16, w [N_rows, K] bf16 (rows contiguous). epi: 0 store, 1 residual, 3 RoPE,
// 4 SwiGLU (w = [gate; up], pair_offset = rows of gate). out: [M, N_out] bf16.
void skinny_linear(const at::Tensor& x, const at::Tensor& w, int64_t epi, const at::Tensor& out,
                   const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& positions,
                   const c10::optional<at::Tensor>& cos_tab, const c10::optional<at::Tensor>& sin_tab,
                   int64_t rope_begin, int64_t rope_end, int64_t pair_offset) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && out.is_cuda(), "skinny_linear: CUDA tensors");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16,
              "skinny_linear: bf16");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1 && out.stride(1) == 1,
              "skinny_linear: row-major operands");
  const int M = (int)x.size(0), K = (int)x.size(1);
  TORCH_CHECK(M >= 1 && M <= SK_MAXM, "skinny_linear: 1 <= M <= 32");
  TORCH_CHECK(w.size(1) == K && K % 8 == 0 && x.stride(0) % 8 == 0 && w.stride(0) % 8 == 0 &&
                  (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(w.data_ptr()) & 15) == 0,
              "skinny_linear: K and row strides must be multiples of 8, bases 16-byte aligned");
  c10::cuda::CUDAGuard guard(x.device());
  SkinnyArgs a{};
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.ldx = x.stride(0);
  a.w = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  a.ldw = w.stride(0);
  a.M = M;
  a.K = K;
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ldo = out.stride(0);
  a.rope_begin = (int)rope_begin;
  a.rope_end = (int)rope_end;
  a.pair_offset = (int)pair_offset;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (epi == SK_SWIGLU) {
    TORCH_CHECK(w.size(0) == 2 * pair_offset && out.size(1) == pair_offset, "skinny_linear: SwiGLU shapes");
    a.pairs = (int)pair_offset;
    return launch_skinny<SK_SWIGLU>(a, stream);
  }
  const int N = (int)w.size(0);
  TORCH_CHECK(out.size(1) == N && N % 2 == 0 && a.ldo % 2 == 0, "skinny_linear: output width");
  a.pairs = N / 2;
  if (epi == SK_ROPE) {
    TORCH_CHECK(N % 128 == 0 && positions && cos_tab && sin_tab, "skinny_linear: RoPE needs 128-wide heads and tables");
    a.positions = positions->data_ptr<int>();
    a.cos_tab = cos_tab->data_ptr<float>();
    a.sin_tab = sin_tab->data_ptr<float>();
    return launch_skinny<SK_ROPE>(a, stream);
  }
  if (epi == SK_RESIDUAL) {
    TORCH_CHECK(residual && residual->stride(1) == 1 && residual->stride(0) % 2 == 0, "skinny_linear: residual");
    a.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    a.ldr = residual->stride(0);
    return launch_skinny<SK_RESIDUAL>(a, stream);
  }
  TORCH_CHECK(epi == SK_STORE, "skinny_linear: unsupported epilogue ", epi);
  launch_skinny<SK_STORE>(a, stream);
}

}  // namespace hrm
