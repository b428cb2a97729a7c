// Memory-bound kernels of the training step (sm_100a): fused add + RMSNorm forward and
// backward, scaled embedding forward/backward, cross-entropy finalisation, in-place
// logits -> dlogits, and the fused AdamATan2 update over flat fp32 buffers.
//
// Rows are processed one warp per row with 16-byte vector accesses; the row width is a
// multiple of 256 elements (8 per lane per chunk) and kept in registers.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace hrm {
at::Tensor device_error_word();
}  // namespace hrm

namespace hrm {

namespace {

__device__ __forceinline__ void unpack8(const uint4& w, float (&v)[8]) {
  const float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), c = unpack_bf16x2(w.z), d = unpack_bf16x2(w.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                    pack_bf16x2(v[6], v[7]));
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffff, x, o);
  return x;
}

// ---------------------------------------------------------------------------------------
// RMSNorm (no weight): s = bf16(x + inj); y = bf16(s * rsqrt(mean(s^2) + eps)).
// x may be broadcast over rows (ldx = 0). s is written when `s_out` is given.
// ---------------------------------------------------------------------------------------
template <int NC>
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, long ldx, const __nv_bfloat16* __restrict__ inj,
                                   long ldi, __nv_bfloat16* __restrict__ s_out, long lds, __nv_bfloat16* __restrict__ y,
                                   long ldy, float* __restrict__ rstd, int T, float eps) {
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  constexpr int H = NC * 256;
  float v[NC][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * 8;
    unpack8(*reinterpret_cast<const uint4*>(x + (long)row * ldx + col), v[c]);
    if (inj != nullptr) {
      float w[8];
      unpack8(*reinterpret_cast<const uint4*>(inj + (long)row * ldi + col), w);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[c][k] = bf16_round(v[c][k] + w[k]);
      if (s_out != nullptr) *reinterpret_cast<uint4*>(s_out + (long)row * lds + col) = pack8(v[c]);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) ss += v[c][k] * v[c][k];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)H + eps);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * 8;
    float o[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = v[c][k] * r;
    *reinterpret_cast<uint4*>(y + (long)row * ldy + col) = pack8(o);
  }
  if (lane == 0 && rstd != nullptr) rstd[row] = r;
}

// dx = rstd * (dy - xhat * mean(dy * xhat)) (+ dres), xhat = s * rstd.
template <int NC>
__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, long lddy, const __nv_bfloat16* __restrict__ s,
                                   long lds, const float* __restrict__ rstd, const __nv_bfloat16* __restrict__ dres,
                                   long ldr, __nv_bfloat16* __restrict__ dx, long lddx, int T) {
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  constexpr int H = NC * 256;
  const float r = rstd[row];
  float g[NC][8], xh[NC][8];
  float dot = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * 8;
    unpack8(*reinterpret_cast<const uint4*>(dy + (long)row * lddy + col), g[c]);
    unpack8(*reinterpret_cast<const uint4*>(s + (long)row * lds + col), xh[c]);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      xh[c][k] *= r;
      dot += g[c][k] * xh[c][k];
    }
  }
  dot = warp_sum(dot) / (float)H;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * 8;
    float o[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = r * (g[c][k] - xh[c][k] * dot);
    if (dres != nullptr) {
      float w[8];
      unpack8(*reinterpret_cast<const uint4*>(dres + (long)row * ldr + col), w);
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] += w[k];
    }
    *reinterpret_cast<uint4*>(dx + (long)row * lddx + col) = pack8(o);
  }
}

// ---------------------------------------------------------------------------------------
// Embedding: out[t] = bf16(scale * W[id[t]]); grad: gW[id[t]] += scale * dout[t] (fp32).
// ---------------------------------------------------------------------------------------
__global__ void embedding_fwd_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ w, long ldw,
                                     __nv_bfloat16* __restrict__ out, long ldo, int T, int H, float scale, int V,
                                     int* err) {
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const long id = ids[row];
  if (!HRM_BOUNDS_OK(id >= 0 && id < V, err, 95)) return;
  for (int col = lane * 8; col < H; col += 256) {
    float v[8];
    unpack8(*reinterpret_cast<const uint4*>(w + id * ldw + col), v);
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] *= scale;
    *reinterpret_cast<uint4*>(out + (long)row * ldo + col) = pack8(v);
  }
}

__global__ void embedding_bwd_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ dout, long ldo,
                                     float* __restrict__ gw, long ldg, int T, int H, float scale, int V, int* err) {
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const long id = ids[row];
  if (!HRM_BOUNDS_OK(id >= 0 && id < V, err, 96)) return;
  for (int col = lane * 8; col < H; col += 256) {
    float v[8];
    unpack8(*reinterpret_cast<const uint4*>(dout + (long)row * ldo + col), v);
    float4* dst = reinterpret_cast<float4*>(gw + id * ldg + col);
    atomicAdd(dst, make_float4(v[0] * scale, v[1] * scale, v[2] * scale, v[3] * scale));
    atomicAdd(dst + 1, make_float4(v[4] * scale, v[5] * scale, v[6] * scale, v[7] * scale));
  }
}

// ---------------------------------------------------------------------------------------
// Cross-entropy: combine per-tile partials -> lse, per-row loss, correctness.
// ---------------------------------------------------------------------------------------
__global__ void ce_finalize_kernel(const float* __restrict__ pmax, const float* __restrict__ psum,
                                   const int* __restrict__ parg, const float* __restrict__ tgt,
                                   const int* __restrict__ labels, int T, int n_tiles, float* __restrict__ lse,
                                   float* __restrict__ loss_rows, uint8_t* __restrict__ correct) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= T) return;
  float gmax = -INFINITY;
  int garg = 0;
  for (int t = 0; t < n_tiles; ++t) {
    const float m = pmax[(long)t * T + row];
    if (m > gmax) {
      gmax = m;
      garg = parg[(long)t * T + row];
    }
  }
  float sum = 0.f;
  for (int t = 0; t < n_tiles; ++t) sum += psum[(long)t * T + row] * __expf(pmax[(long)t * T + row] - gmax);
  const float l = gmax + __logf(sum);
  lse[row] = l;
  const int label = labels[row];
  const bool valid = label >= 0;
  loss_rows[row] = valid ? (l - tgt[row]) : 0.f;
  correct[row] = (valid && garg == label) ? 1 : 0;
}

// logits (bf16, in place) -> (softmax - onehot) * grad for valid rows, 0 otherwise.
__global__ void ce_dlogits_kernel(__nv_bfloat16* __restrict__ logits, long ld, const float* __restrict__ lse,
                                  const int* __restrict__ labels, const float* __restrict__ grad, int T, int V) {
  const long chunks_per_row = V / 8;
  const float g = *grad;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < (long)T * chunks_per_row;
       i += (long)gridDim.x * blockDim.x) {
    const long row = i / chunks_per_row;
    const int col = (int)(i % chunks_per_row) * 8;
    const int label = labels[row];
    uint4* p = reinterpret_cast<uint4*>(logits + row * ld + col);
    if (label < 0) {
      *p = make_uint4(0, 0, 0, 0);
      continue;
    }
    const float l = lse[row];
    float v[8];
    unpack8(*p, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float prob = __expf(v[k] - l);
      v[k] = (prob - (col + k == label ? 1.f : 0.f)) * g;
    }
    *p = pack8(v);
  }
}

// ---------------------------------------------------------------------------------------
// AdamATan2 over flat fp32 buffers. hyper (device): [lr, 1/(1-b1^t), 1/sqrt(1-b2^t)].
// ---------------------------------------------------------------------------------------
__global__ void adam_atan2_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                                  float* __restrict__ v, float* __restrict__ ema, __nv_bfloat16* __restrict__ out16,
                                  long n, const float* __restrict__ hyper, float beta1, float beta2, float wd,
                                  float ema_decay) {
  const float lr = hyper[0], inv_bc1 = hyper[1], inv_bc2_sqrt = hyper[2];
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    float vv = v[i];
    float mv = m != nullptr ? m[i] : 0.f;
    const float pv = adam_atan2_update(p[i], g[i], m != nullptr, mv, vv, lr, inv_bc1, inv_bc2_sqrt, beta1,
                                       beta2, wd);
    v[i] = vv;
    if (m != nullptr) m[i] = mv;
    p[i] = pv;
    if (ema != nullptr) {
      float e = ema[i];
      e = e + (1.f - ema_decay) * (pv - e);
      ema[i] = e;
    }
    if (out16 != nullptr) out16[i] = __float2bfloat16(pv);
  }
}

// Same update, four parameters per thread with 16-byte loads / stores (all buffers 16-byte
// aligned, n a multiple of 4): the optimizer moves ~38 bytes per parameter, so it is bound by
// HBM bandwidth and the scalar version left a third of it unused.
__global__ void adam_atan2_vec4_kernel(float4* __restrict__ p, const float4* __restrict__ g, float4* __restrict__ m,
                                       float4* __restrict__ v, float4* __restrict__ ema, uint2* __restrict__ out16,
                                       long n4, const float* __restrict__ hyper, float beta1, float beta2, float wd,
                                       float ema_decay) {
  const float lr = hyper[0], inv_bc1 = hyper[1], inv_bc2_sqrt = hyper[2];
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    float4 pv = p[i], gv = g[i], vv = v[i];
    float4 mv = m != nullptr ? m[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    float* pp = &pv.x; const float* gg = &gv.x; float* vp = &vv.x; float* mp = &mv.x;
#pragma unroll
    for (int e = 0; e < 4; ++e)
      pp[e] = adam_atan2_update(pp[e], gg[e], m != nullptr, mp[e], vp[e], lr, inv_bc1, inv_bc2_sqrt, beta1, beta2, wd);
    p[i] = pv;
    v[i] = vv;
    if (m != nullptr) m[i] = mv;
    if (ema != nullptr) {
      float4 e = ema[i];
      const float d = 1.f - ema_decay;
      e.x += d * (pv.x - e.x); e.y += d * (pv.y - e.y); e.z += d * (pv.z - e.z); e.w += d * (pv.w - e.w);
      ema[i] = e;
    }
    if (out16 != nullptr) out16[i] = make_uint2(pack_bf16x2(pv.x, pv.y), pack_bf16x2(pv.z, pv.w));
  }
}

__global__ void cast_f32_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, long n) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    dst[i] = __float2bfloat16(src[i]);
}

int grid_for(long n, int threads, int max_blocks = 148 * 16) {
  long b = (n + threads - 1) / threads;
  return (int)std::max<long>(1, std::min<long>(b, max_blocks));
}

}  // namespace

// ---------------------------------------------------------------------------------------
// host API
// ---------------------------------------------------------------------------------------
#define HRM_NC_DISPATCH(NC_VAL, ...)                                     \
  switch (NC_VAL) {                                                      \
    case 1: { constexpr int NC = 1; __VA_ARGS__; break; }                \
    case 2: { constexpr int NC = 2; __VA_ARGS__; break; }                \
    case 3: { constexpr int NC = 3; __VA_ARGS__; break; }                \
    case 4: { constexpr int NC = 4; __VA_ARGS__; break; }                \
    case 5: { constexpr int NC = 5; __VA_ARGS__; break; }                \
    case 6: { constexpr int NC = 6; __VA_ARGS__; break; }                \
    case 7: { constexpr int NC = 7; __VA_ARGS__; break; }                \
    case 8: { constexpr int NC = 8; __VA_ARGS__; break; }                \
    case 10: { constexpr int NC = 10; __VA_ARGS__; break; }              \
    case 12: { constexpr int NC = 12; __VA_ARGS__; break; }              \
    default: TORCH_CHECK(false, "row width must be 256 * {1..8,10,12}"); \
  }

static const __nv_bfloat16* bf(const at::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); }
static __nv_bfloat16* bfm(const at::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }

void rmsnorm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& inj, const c10::optional<at::Tensor>& s_out,
                 const at::Tensor& y, const at::Tensor& rstd, int64_t T, double eps) {
  c10::cuda::CUDAGuard guard(y.device());
  const int H = (int)y.size(-1);
  TORCH_CHECK(H % 256 == 0, "rmsnorm width must be a multiple of 256");
  const long ldx = (x.dim() == 1) ? 0 : x.stride(0);
  const int rows_per_block = 8;
  const int blocks = (int)((T + rows_per_block - 1) / rows_per_block);
  auto stream = at::cuda::getCurrentCUDAStream();
  HRM_NC_DISPATCH(H / 256, rmsnorm_fwd_kernel<NC><<<blocks, rows_per_block * 32, 0, stream>>>(
                               bf(x), ldx, inj ? bf(*inj) : nullptr, inj ? inj->stride(0) : 0,
                               s_out ? bfm(*s_out) : nullptr, s_out ? s_out->stride(0) : 0, bfm(y), y.stride(0),
                               rstd.numel() ? rstd.data_ptr<float>() : nullptr, (int)T, (float)eps));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& s, const at::Tensor& rstd,
                 const c10::optional<at::Tensor>& dres, const at::Tensor& dx, int64_t T) {
  c10::cuda::CUDAGuard guard(dy.device());
  const int H = (int)dy.size(-1);
  const int rows_per_block = 8;
  const int blocks = (int)((T + rows_per_block - 1) / rows_per_block);
  auto stream = at::cuda::getCurrentCUDAStream();
  HRM_NC_DISPATCH(H / 256, rmsnorm_bwd_kernel<NC><<<blocks, rows_per_block * 32, 0, stream>>>(
                               bf(dy), dy.stride(0), bf(s), s.stride(0), rstd.data_ptr<float>(),
                               dres ? bf(*dres) : nullptr, dres ? dres->stride(0) : 0, bfm(dx), dx.stride(0), (int)T));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embedding_fwd(const at::Tensor& ids, const at::Tensor& w, const at::Tensor& out, double scale) {
  c10::cuda::CUDAGuard guard(w.device());
  const int T = (int)ids.numel(), H = (int)w.size(1);
  TORCH_CHECK(H % 8 == 0, "embedding width must be a multiple of 8");
  embedding_fwd_kernel<<<(T + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int>(), bf(w), w.stride(0), bfm(out), out.stride(0), T, H, (float)scale, (int)w.size(0),
      device_error_word().data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embedding_bwd(const at::Tensor& ids, const at::Tensor& dout, const at::Tensor& gw, double scale) {
  c10::cuda::CUDAGuard guard(dout.device());
  const int T = (int)ids.numel(), H = (int)dout.size(1);
  embedding_bwd_kernel<<<(T + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int>(), bf(dout), dout.stride(0), gw.data_ptr<float>(), gw.stride(0), T, H, (float)scale,
      (int)gw.size(0), device_error_word().data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ce_finalize(const at::Tensor& pmax, const at::Tensor& psum, const at::Tensor& parg, const at::Tensor& tgt,
                 const at::Tensor& labels, const at::Tensor& lse, const at::Tensor& loss_rows,
                 const at::Tensor& correct) {
  c10::cuda::CUDAGuard guard(labels.device());
  const int T = (int)labels.numel(), n_tiles = (int)pmax.size(0);
  ce_finalize_kernel<<<(T + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      pmax.data_ptr<float>(), psum.data_ptr<float>(), parg.data_ptr<int>(), tgt.data_ptr<float>(),
      labels.data_ptr<int>(), T, n_tiles, lse.data_ptr<float>(), loss_rows.data_ptr<float>(),
      correct.data_ptr<uint8_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ce_dlogits(const at::Tensor& logits, const at::Tensor& lse, const at::Tensor& labels, const at::Tensor& grad) {
  c10::cuda::CUDAGuard guard(logits.device());
  const int T = (int)logits.size(0), V = (int)logits.size(1);
  TORCH_CHECK(V % 8 == 0, "vocab must be a multiple of 8");
  const long n = (long)T * (V / 8);
  ce_dlogits_kernel<<<grid_for(n, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      bfm(logits), logits.stride(0), lse.data_ptr<float>(), labels.data_ptr<int>(), grad.data_ptr<float>(), T, V);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void adam_atan2(const at::Tensor& p, const at::Tensor& g, const c10::optional<at::Tensor>& m, const at::Tensor& v,
                const c10::optional<at::Tensor>& ema, const c10::optional<at::Tensor>& out16, const at::Tensor& hyper,
                double beta1, double beta2, double wd, double ema_decay) {
  c10::cuda::CUDAGuard guard(p.device());
  const long n = p.numel();
  TORCH_CHECK(g.numel() == n && v.numel() == n, "adam_atan2: size mismatch");
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  const bool vec = n % 4 == 0 && a16(p.data_ptr()) && a16(g.data_ptr()) && a16(v.data_ptr()) &&
                   (!m || a16(m->data_ptr())) && (!ema || a16(ema->data_ptr())) &&
                   (!out16 || (reinterpret_cast<uintptr_t>(out16->data_ptr()) & 7) == 0);
  if (vec) {
    adam_atan2_vec4_kernel<<<grid_for(n / 4, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<float4*>(p.data_ptr<float>()), reinterpret_cast<const float4*>(g.data_ptr<float>()),
        m ? reinterpret_cast<float4*>(m->data_ptr<float>()) : nullptr, reinterpret_cast<float4*>(v.data_ptr<float>()),
        ema ? reinterpret_cast<float4*>(ema->data_ptr<float>()) : nullptr,
        out16 ? reinterpret_cast<uint2*>(out16->data_ptr()) : nullptr, n / 4, hyper.data_ptr<float>(), (float)beta1,
        (float)beta2, (float)wd, (float)ema_decay);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  adam_atan2_kernel<<<grid_for(n, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      p.data_ptr<float>(), g.data_ptr<float>(), m ? m->data_ptr<float>() : nullptr, v.data_ptr<float>(),
      ema ? ema->data_ptr<float>() : nullptr, out16 ? bfm(*out16) : nullptr, n, hyper.data_ptr<float>(),
      (float)beta1, (float)beta2, (float)wd, (float)ema_decay);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void cast_f32_bf16(const at::Tensor& src, const at::Tensor& dst) {
  c10::cuda::CUDAGuard guard(src.device());
  const long n = src.numel();
  cast_f32_bf16_kernel<<<grid_for(n, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(src.data_ptr<float>(),
                                                                                      bfm(dst), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------------------
// device error word: 4 x int32 per device, zero until a kernel reports a bounded-wait
// timeout (code, site, block, thread).
// ---------------------------------------------------------------------------------------
// True when the extension was built with HRM_DEBUG_BOUNDS (device-side bounds checks).
bool debug_bounds_build() { return kDebugBounds; }

at::Tensor device_error_word() {
  static at::Tensor* words = new at::Tensor[16];  // intentionally leaked: no teardown after the driver
  int dev;
  cudaGetDevice(&dev);
  TORCH_CHECK(dev < 16, "too many devices");
  if (!words[dev].defined())
    words[dev] = at::zeros({4}, at::TensorOptions().dtype(at::kInt).device(at::kCUDA, dev));
  return words[dev];
}

}  // namespace hrm
