// KV-cache attention for decoding: one new query per sequence against its cached keys.
//
// Counterpart of the reference's flash_attn_with_kvcache call in decode mode
// (models/layers.py:148-151; inference in simple_inference_engine.py:105-112): query b, head h
// attends to cache positions [0, total[b]) of k_cache / v_cache ([B, S_max, H, 128] bf16, any
// row strides), where total[b] already counts the key appended for this step.
//
// Split-KV ("flash-decoding"): grid (splits, B*H); each CTA owns one key range of one
// (sequence, head); its 4 warps stream keys (each lane holds 4 of the 128 dims, so a key row is
// one coalesced 256-byte warp load), keep an online softmax in the log2 domain, and are merged
// through shared memory. With one split the CTA writes the bf16 output; otherwise it writes a
// (max, sum, o[128]) partial and decode_combine_kernel merges the splits. Decoding is bound by
// reading the cache, so CUDA cores at full memory bandwidth are the right tool (M = 1).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "device_setup.h"

namespace hrm {
at::Tensor device_error_word();
namespace {

constexpr int D = 128;
constexpr int WARPS = 8;
constexpr int KG = 4;  // keys per warp iteration: their loads are in flight together

__device__ __forceinline__ void load4(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 w = *reinterpret_cast<const uint2*>(p);
  const float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}

__global__ void __launch_bounds__(WARPS * 32)
    decode_split_kernel(const __nv_bfloat16* __restrict__ q, long q_sb, long q_sh, const __nv_bfloat16* __restrict__ kc,
                        const __nv_bfloat16* __restrict__ vc, long c_sb, long c_ss, long c_sh,
                        const int* __restrict__ total, int total_offset, int S_max, int* err, int H, int chunk,
                        float scale_log2,
                        const __nv_bfloat16* __restrict__ gate, long g_sb, long g_sh,
                        __nv_bfloat16* __restrict__ out, long o_sb, long o_sh, float* __restrict__ part) {
  __shared__ float sm[WARPS], sl[WARPS];
  __shared__ float so[WARPS][D];
  const int split = blockIdx.x, splits = gridDim.x;
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int n = total[b] + total_offset;
  if (!HRM_BOUNDS_OK(n >= 0 && n <= S_max, err, 90)) n = max(0, min(n, S_max));
  const int c0 = split * chunk, c1 = min(n, c0 + chunk);

  float qv[4];
  load4(q + b * q_sb + h * q_sh + lane * 4, qv);
#pragma unroll
  for (int i = 0; i < 4; ++i) qv[i] *= scale_log2;
  float m = -INFINITY, l = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
  const __nv_bfloat16* kb = kc + b * c_sb + h * c_sh + lane * 4;
  const __nv_bfloat16* vb = vc + b * c_sb + h * c_sh + lane * 4;
  // KG keys per iteration: all their K / V rows are requested before any is used (decoding is
  // bound by the latency of these loads, not by arithmetic)
  for (int j0 = c0 + warp * KG; j0 < c1; j0 += WARPS * KG) {
    float kv[KG][4], vv[KG][4], sc[KG];
#pragma unroll
    for (int u = 0; u < KG; ++u) {
      const int j = min(j0 + u, c1 - 1);  // clamped: the duplicate is masked below
      load4(kb + (long)j * c_ss, kv[u]);
      load4(vb + (long)j * c_ss, vv[u]);
    }
#pragma unroll
    for (int u = 0; u < KG; ++u) sc[u] = qv[0] * kv[u][0] + qv[1] * kv[u][1] + qv[2] * kv[u][2] + qv[3] * kv[u][3];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int u = 0; u < KG; ++u) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], off);
    float m_new = m;
#pragma unroll
    for (int u = 0; u < KG; ++u) {
      if (j0 + u >= c1) sc[u] = -INFINITY;
      m_new = fmaxf(m_new, sc[u]);
    }
    const float alpha = fast_exp2(m - m_new);  // 0 on the first keys (m = -inf)
    l *= alpha;
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] *= alpha;
#pragma unroll
    for (int u = 0; u < KG; ++u) {
      const float p = fast_exp2(sc[u] - m_new);  // 0 for masked keys
      l += p;
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = fmaf(p, vv[u][i], o[i]);
    }
    m = m_new;
  }
  if (lane == 0) {
    sm[warp] = m;
    sl[warp] = l;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) so[warp][lane * 4 + i] = o[i];
  __syncthreads();
  // merge the warps: thread t < 128 owns dim t
  const int t = threadIdx.x;
  if (t >= D) return;
  float mm = -INFINITY;
#pragma unroll
  for (int w = 0; w < WARPS; ++w) mm = fmaxf(mm, sm[w]);
  const float ref = mm == -INFINITY ? 0.f : mm;
  float L = 0.f, O = 0.f;
#pragma unroll
  for (int w = 0; w < WARPS; ++w) {
    const float f = fast_exp2(sm[w] - ref);
    L += sl[w] * f;
    O += so[w][t] * f;
  }
  if (splits == 1) {
    float val = bf16_round(L > 0.f ? O / L : 0.f);
    if (gate != nullptr) val *= sigmoidf_(__bfloat162float(gate[b * g_sb + h * g_sh + t]));
    out[b * o_sb + h * o_sh + t] = __float2bfloat16_rn(val);
  } else {
    float* pp = part + ((long)bh * splits + split) * (D + 2);
    pp[2 + t] = O;
    if (t == 0) {
      pp[0] = mm;
      pp[1] = L;
    }
  }
}

__global__ void decode_combine_kernel(const float* __restrict__ part, int splits, int H,
                                      const __nv_bfloat16* __restrict__ gate, long g_sb, long g_sh,
                                      __nv_bfloat16* __restrict__ out, long o_sb, long o_sh) {
  const int bh = blockIdx.x, b = bh / H, h = bh % H, t = threadIdx.x;
  const float* pp = part + (long)bh * splits * (D + 2);
  float mm = -INFINITY;
  for (int s = 0; s < splits; ++s) mm = fmaxf(mm, pp[s * (D + 2)]);
  const float ref = mm == -INFINITY ? 0.f : mm;
  float L = 0.f, O = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float f = fast_exp2(pp[s * (D + 2)] - ref);
    L += pp[s * (D + 2) + 1] * f;
    O += pp[s * (D + 2) + 2 + t] * f;
  }
  float val = bf16_round(L > 0.f ? O / L : 0.f);
  if (gate != nullptr) val *= sigmoidf_(__bfloat162float(gate[b * g_sb + h * g_sh + t]));
  out[b * o_sb + h * o_sh + t] = __float2bfloat16_rn(val);
}

// The decode step's new key / value rows (from the fused gate|q|k|v projection output) into
// the caches at position lengths[b]: one CTA per sequence, 16-byte copies.
__global__ void kv_append_kernel(const __nv_bfloat16* __restrict__ gqkv, long ld, int H, const int* __restrict__ lengths,
                                 __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc, long c_sb, long c_ss,
                                 long c_sh, int S_max, int* err) {
  const int b = blockIdx.x;
  const long pos = lengths[b];
  if (!HRM_BOUNDS_OK(pos >= 0 && pos < S_max, err, 91)) return;
  for (int i = threadIdx.x; i < H * 16; i += blockDim.x) {
    const int h = i >> 4, c = (i & 15) * 8;
    const uint4 k = *reinterpret_cast<const uint4*>(gqkv + b * ld + (long)(2 * H + h) * D + c);
    const uint4 v = *reinterpret_cast<const uint4*>(gqkv + b * ld + (long)(3 * H + h) * D + c);
    *reinterpret_cast<uint4*>(kc + b * c_sb + pos * c_ss + h * c_sh + c) = k;
    *reinterpret_cast<uint4*>(vc + b * c_sb + pos * c_ss + h * c_sh + c) = v;
  }
}

// Key ranges per (sequence, head): about 128 cache positions each (16 per warp), so that the
// loads of all warps together keep enough bytes in flight; a combine pass merges the ranges.
int decode_splits(int B, int H, int S) {
  (void)B;
  (void)H;
  return std::max(1, std::min(64, (S + 127) / 128));
}

}  // namespace

// q [B, H, 128], k_cache / v_cache [B, S_max, H, 128] (bf16, last dim contiguous), total [B]
// int32 visible keys per sequence; returns out [B, H, 128] bf16.
at::Tensor decode_attention(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                            const at::Tensor& total) {
  TORCH_CHECK(q.is_cuda() && q.dim() == 3 && q.size(2) == D && q.stride(2) == 1, "q: [B, H, 128] CUDA");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(3) == D && k_cache.stride(3) == 1 && v_cache.sizes() == k_cache.sizes() &&
                  v_cache.strides() == k_cache.strides(),
              "caches: [B, S_max, H, 128] with matching strides");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k_cache.scalar_type() == at::kBFloat16 &&
                  v_cache.scalar_type() == at::kBFloat16,
              "decode attention is bf16");
  TORCH_CHECK(total.scalar_type() == at::kInt && total.numel() == q.size(0), "total: int32 [B]");
  TORCH_CHECK(q.stride(1) % 4 == 0 && q.stride(0) % 4 == 0 && k_cache.stride(2) % 4 == 0 && k_cache.stride(1) % 4 == 0 &&
                  k_cache.stride(0) % 4 == 0,
              "8-byte aligned rows required");
  c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int B = (int)q.size(0), H = (int)q.size(1), S = (int)k_cache.size(1);
  auto out = at::empty({B, H, D}, q.options());
  // splits: enough CTAs to cover the GPU when B*H is small, one when the cache is short
  const int splits = decode_splits(B, H, S);
  const int chunk = (S + splits - 1) / splits;
  at::Tensor part;
  if (splits > 1) part = at::empty({(long)B * H * splits * (D + 2)}, q.options().dtype(at::kFloat));
  const float scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)D));
  decode_split_kernel<<<dim3(splits, B * H), WARPS * 32, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), q.stride(0), q.stride(1),
      reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr()),
      k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), total.data_ptr<int>(), 0, S,
      device_error_word().data_ptr<int>(), H, chunk, scale_log2,
      nullptr, 0, 0, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), out.stride(1),
      splits > 1 ? part.data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (splits > 1) {
    decode_combine_kernel<<<B * H, D, 0, stream>>>(part.data_ptr<float>(), splits, H, nullptr, 0, 0,
                                                   reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0),
                                                   out.stride(1));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return out;
}

// The whole attention of one decode step from the fused projection output gqkv [B, 4H*128]
// (gate, q, k, v heads; q and k rotated): appends k / v at lengths[b] in the caches, attends
// over [0, lengths[b] + 1) and returns y = sigmoid(gate) * O as [B, H*128] bf16.
at::Tensor decode_attention_gqkv(const at::Tensor& gqkv, int64_t H, const at::Tensor& k_cache,
                                 const at::Tensor& v_cache, const at::Tensor& lengths) {
  TORCH_CHECK(gqkv.is_cuda() && gqkv.dim() == 2 && gqkv.size(1) >= 4 * H * D && gqkv.stride(1) == 1 &&
                  gqkv.scalar_type() == at::kBFloat16 && gqkv.stride(0) % 8 == 0,
              "gqkv: [B, 4*H*128] bf16 with 16-byte aligned rows");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(2) == H && k_cache.size(3) == D && k_cache.stride(3) == 1 &&
                  v_cache.sizes() == k_cache.sizes() && v_cache.strides() == k_cache.strides() &&
                  k_cache.scalar_type() == at::kBFloat16 && v_cache.scalar_type() == at::kBFloat16 &&
                  k_cache.stride(2) % 8 == 0 && k_cache.stride(1) % 8 == 0 && k_cache.stride(0) % 8 == 0,
              "caches: [B, S_max, H, 128] bf16 with matching, 16-byte aligned strides");
  TORCH_CHECK(lengths.scalar_type() == at::kInt && lengths.numel() == gqkv.size(0), "lengths: int32 [B]");
  c10::cuda::CUDAGuard guard(gqkv.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int B = (int)gqkv.size(0), S = (int)k_cache.size(1), h = (int)H;
  const long ld = gqkv.stride(0);
  auto kc = reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr());
  auto vc = reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr());
  const auto* g = reinterpret_cast<const __nv_bfloat16*>(gqkv.data_ptr());
  kv_append_kernel<<<B, 256, 0, stream>>>(g, ld, h, lengths.data_ptr<int>(), kc, vc, k_cache.stride(0),
                                          k_cache.stride(1), k_cache.stride(2), S, device_error_word().data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  auto out = at::empty({B, h * D}, gqkv.options());
  const int splits = decode_splits(B, h, S);
  const int chunk = (S + splits - 1) / splits;
  at::Tensor part;
  if (splits > 1) part = at::empty({(long)B * h * splits * (D + 2)}, gqkv.options().dtype(at::kFloat));
  const float scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)D));
  auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  decode_split_kernel<<<dim3(splits, B * h), WARPS * 32, 0, stream>>>(
      g + (long)h * D, ld, D, kc, vc, k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
      lengths.data_ptr<int>(), 1, S, device_error_word().data_ptr<int>(), h, chunk, scale_log2, g, ld, D, o,
      out.stride(0), D,
      splits > 1 ? part.data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (splits > 1) {
    decode_combine_kernel<<<B * h, D, 0, stream>>>(part.data_ptr<float>(), splits, h, g, ld, D, o, out.stride(0), D);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return out;
}

}  // namespace hrm
