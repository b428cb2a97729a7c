// Token sampling for generation: greedy argmax or Gumbel-max at a temperature, one CTA per
// row of logits, fused (scale, noise, argmax) in a single pass over the vocabulary.
//
// Same rule as the reference (simple_inference_engine.py:93-102): argmax(logits) when
// temp < 1e-5, else argmax(logits / temp - log(-log u)) with u ~ U(0, 1). The uniforms come
// from a counter-based generator: SplitMix64 (Steele, Lea, Flood, "Fast splittable pseudorandom
// number generators", OOPSLA 2014) applied to (seed, offset, row, column), so a call is
// reproducible from (seed, offset) and needs no generator state on the device.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace hrm {
namespace {

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// lexicographic (value descending, index ascending): the first maximum wins, as torch.argmax
__device__ __forceinline__ void better(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}

template <typename T>
__global__ void __launch_bounds__(512) sample_kernel(const T* __restrict__ logits, long ld, int V, float inv_temp,
                                                     int greedy, uint64_t seed, uint64_t offset,
                                                     int64_t* __restrict__ out) {
  const int row = blockIdx.x;
  const T* x = logits + (long)row * ld;
  float best = -INFINITY;
  int best_i = 0x7fffffff;
  const uint64_t key = splitmix64(seed ^ splitmix64(offset + 0x632BE59BD9B4E019ull * (uint64_t)(row + 1)));
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    float v = to_f(x[j]);
    if (!greedy) {
      // 24 random bits -> u in (0, 1): never 0, never 1
      const uint32_t bits = (uint32_t)(splitmix64(key + (uint64_t)j) >> 40);
      const float u = ((float)bits + 0.5f) * (1.0f / 16777216.0f);
      v = v * inv_temp - logf(-logf(u));
    }
    better(best, best_i, v, j);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, best, off);
    const int i2 = __shfl_xor_sync(0xffffffffu, best_i, off);
    better(best, best_i, v2, i2);
  }
  __shared__ float sv[16];
  __shared__ int si[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = best_i;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -INFINITY;
    best_i = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float v2 = __shfl_xor_sync(0xffffffffu, best, off);
      const int i2 = __shfl_xor_sync(0xffffffffu, best_i, off);
      better(best, best_i, v2, i2);
    }
    if (lane == 0) out[row] = best_i == 0x7fffffff ? 0 : best_i;
  }
}

}  // namespace

// logits [B, V] (fp32 or bf16, rows contiguous) -> int64 [B] token ids.
at::Tensor sample_tokens(const at::Tensor& logits, double temp, int64_t seed, int64_t offset) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.stride(1) == 1, "logits: CUDA [B, V], rows contiguous");
  c10::cuda::CUDAGuard guard(logits.device());
  const int B = (int)logits.size(0), V = (int)logits.size(1);
  auto out = at::empty({B}, logits.options().dtype(at::kLong));
  if (B == 0) return out;
  const bool greedy = temp < 1e-5;
  const float inv_temp = greedy ? 1.f : (float)(1.0 / temp);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (logits.scalar_type() == at::kFloat) {
    sample_kernel<float><<<B, 512, 0, stream>>>(logits.data_ptr<float>(), logits.stride(0), V, inv_temp, greedy,
                                                (uint64_t)seed, (uint64_t)offset, out.data_ptr<int64_t>());
  } else {
    TORCH_CHECK(logits.scalar_type() == at::kBFloat16, "logits must be fp32 or bf16");
    sample_kernel<__nv_bfloat16><<<B, 512, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()),
                                                        logits.stride(0), V, inv_temp, greedy, (uint64_t)seed,
                                                        (uint64_t)offset, out.data_ptr<int64_t>());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

}  // namespace hrm
