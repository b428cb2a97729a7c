// Small-M linear layers for the decode step (M = sequences being decoded, at most 128).
//
// At small M a linear layer is bound by streaming W once from HBM. The tcgen05 GEMM
// (gemm_tcgen05.cu) with whole 128 x 256 output tiles would give only N / 256 CTAs, so the
// decode path runs it in its split-K mode instead: K is cut into ranges spread over all SMs,
// the unit of K range q stores its fp32 partial tile into slice q of a [split, M, N] buffer
// (plain stores, no atomics, nothing to zero), and this file's finishing kernel sums the
// slices in order -- so a decode step is bit-reproducible -- and turns the sum into the
// layer's bf16 output with the training GEMM's epilogues:
//   EPI_STORE / EPI_RESIDUAL  bf16(acc) (+ bf16 residual)
//   EPI_ROPE                  rotate-half RoPE at positions[m] on the q / k heads in
//                             [rope_begin, rope_end) (pairs 128h + i, 128h + i + 64)
//   EPI_SWIGLU                h = silu(gate) * up with gate = acc[:, f], up = acc[:, f + pair_offset]
// Values are rounded to bf16 before the epilogue math, as the reference rounds the projection
// output.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace hrm {
namespace {

enum DecodeEpi : int { DE_STORE = 0, DE_RESIDUAL = 1, DE_ROPE = 3, DE_SWIGLU = 4 };

struct FinishArgs {
  const float* acc;  // [nsplit][M, N] fp32: row stride lda, slice stride slice
  long lda, slice;
  int nsplit;
  int M, n_out;      // outputs per row
  __nv_bfloat16* out;
  long ldo;
  const __nv_bfloat16* residual;
  long ldr;
  const int* positions;
  const float* cos_tab;  // [max_pos, 64]
  const float* sin_tab;
  int rope_begin, rope_end, pair_offset;
};

__device__ __forceinline__ float slice_sum(const FinishArgs& a, long idx) {
  float v = 0.f;
  for (int q = 0; q < a.nsplit; ++q) v += a.acc[q * a.slice + idx];  // fixed order
  return v;
}
__device__ __forceinline__ float2 slice_sum2(const FinishArgs& a, long idx) {
  float2 v = make_float2(0.f, 0.f);
  for (int q = 0; q < a.nsplit; ++q) {
    const float2 t = *reinterpret_cast<const float2*>(a.acc + q * a.slice + idx);
    v.x += t.x;
    v.y += t.y;
  }
  return v;
}

// One thread per output pair (two adjacent outputs of a row; for RoPE the rotate-half pair).
template <int EPI>
__global__ void decode_finish_kernel(const FinishArgs a) {
  const int pairs_per_row = a.n_out / 2;
  const long total = (long)a.M * pairs_per_row;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int m = (int)(i / pairs_per_row), p = (int)(i % pairs_per_row);
    const long arow = (long)m * a.lda;
    __nv_bfloat16* orow = a.out + (long)m * a.ldo;
    if constexpr (EPI == DE_SWIGLU) {
      const int f = 2 * p;  // outputs f, f + 1
      const float2 g = slice_sum2(a, arow + f);
      const float2 u = slice_sum2(a, arow + a.pair_offset + f);
      const float g0 = bf16_round(g.x), g1 = bf16_round(g.y), u0 = bf16_round(u.x), u1 = bf16_round(u.y);
      const float h0 = __fdividef(g0, 1.0f + __expf(-g0)) * u0;  // fast divide: the output is bf16
      const float h1 = __fdividef(g1, 1.0f + __expf(-g1)) * u1;
      *reinterpret_cast<uint32_t*>(orow + f) = pack_bf16x2(h0, h1);
    } else if constexpr (EPI == DE_ROPE) {
      const int f0 = (p >> 6) * 128 + (p & 63), f1 = f0 + 64;
      float v0 = bf16_round(slice_sum(a, arow + f0)), v1 = bf16_round(slice_sum(a, arow + f1));
      if (f0 >= a.rope_begin && f0 < a.rope_end) {
        const long pos = a.positions[m];
        const float c = a.cos_tab[pos * 64 + (f0 & 63)], s = a.sin_tab[pos * 64 + (f0 & 63)];
        const float r0 = v0 * c - v1 * s, r1 = v1 * c + v0 * s;
        v0 = r0;
        v1 = r1;
      }
      orow[f0] = __float2bfloat16_rn(v0);
      orow[f1] = __float2bfloat16_rn(v1);
    } else {
      const int f = 2 * p;
      const float2 v = slice_sum2(a, arow + f);
      float v0 = bf16_round(v.x), v1 = bf16_round(v.y);
      if constexpr (EPI == DE_RESIDUAL) {
        const float2 r = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(a.residual + (long)m * a.ldr + f));
        v0 += r.x;
        v1 += r.y;
      }
      *reinterpret_cast<uint32_t*>(orow + f) = pack_bf16x2(v0, v1);
    }
  }
}

template <int EPI>
void launch_finish(const FinishArgs& a, cudaStream_t stream) {
  const long total = (long)a.M * (a.n_out / 2);
  const int blocks = (int)std::max<long>(1, std::min<long>((total + 255) / 256, 4096));
  decode_finish_kernel<EPI><<<blocks, 256, 0, stream>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace

// acc [split, M, N] fp32 (the split-K GEMM's slices); out [M, N] bf16 (N / 2 for SwiGLU, where
// pair_offset = N / 2). epi: 0 store, 1 residual, 3 RoPE, 4 SwiGLU.
void decode_linear_finish(const at::Tensor& acc, int64_t epi, const at::Tensor& out,
                          const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& positions,
                          const c10::optional<at::Tensor>& cos_tab, const c10::optional<at::Tensor>& sin_tab,
                          int64_t rope_begin, int64_t rope_end, int64_t pair_offset) {
  TORCH_CHECK(acc.is_cuda() && out.is_cuda() && acc.scalar_type() == at::kFloat && out.scalar_type() == at::kBFloat16,
              "decode_linear_finish: fp32 accumulator, bf16 output");
  TORCH_CHECK(acc.dim() == 3 && out.dim() == 2 && acc.stride(2) == 1 && out.stride(1) == 1 && acc.stride(1) % 2 == 0 &&
                  acc.stride(0) % 2 == 0 && out.stride(0) % 2 == 0 && out.size(0) == acc.size(1),
              "decode_linear_finish: [split, M, N] slices and an [M, N'] output with even row strides");
  c10::cuda::CUDAGuard guard(acc.device());
  FinishArgs a{};
  a.acc = acc.data_ptr<float>();
  a.slice = acc.stride(0);
  a.nsplit = (int)acc.size(0);
  a.lda = acc.stride(1);
  a.M = (int)acc.size(1);
  a.n_out = (int)out.size(1);
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ldo = out.stride(0);
  a.rope_begin = (int)rope_begin;
  a.rope_end = (int)rope_end;
  a.pair_offset = (int)pair_offset;
  TORCH_CHECK(a.n_out % 2 == 0, "decode_linear_finish: even output width");
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (epi == DE_SWIGLU) {
    TORCH_CHECK(acc.size(2) == 2 * pair_offset && a.n_out == pair_offset, "decode_linear_finish: SwiGLU shapes");
    return launch_finish<DE_SWIGLU>(a, stream);
  }
  TORCH_CHECK(acc.size(2) == a.n_out, "decode_linear_finish: output width");
  if (epi == DE_ROPE) {
    TORCH_CHECK(a.n_out % 128 == 0 && positions && cos_tab && sin_tab, "decode_linear_finish: RoPE needs tables");
    a.positions = positions->data_ptr<int>();
    a.cos_tab = cos_tab->data_ptr<float>();
    a.sin_tab = sin_tab->data_ptr<float>();
    return launch_finish<DE_ROPE>(a, stream);
  }
  if (epi == DE_RESIDUAL) {
    TORCH_CHECK(residual && residual->stride(1) == 1 && residual->stride(0) % 2 == 0, "decode_linear_finish: residual");
    a.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    a.ldr = residual->stride(0);
    return launch_finish<DE_RESIDUAL>(a, stream);
  }
  TORCH_CHECK(epi == DE_STORE, "decode_linear_finish: unsupported epilogue ", epi);
  launch_finish<DE_STORE>(a, stream);
}

}  // namespace hrm
