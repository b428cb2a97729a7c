// Step-end update of one rank's parameter shards (multi-GPU sharding engine, fused path).
//
// The gradient of a block weight reaches its owner during the backward: the last weight-
// gradient GEMM of the step (EPI_F2 in gemm_tcgen05.cu) pushes every finished 32 x 128 region
// into the sender's slot of the owner's fp32 inbox and counts it on the owner's 32-row group.
// This kernel, run once per step on every rank, turns that into the optimizer step:
//   for each work item (a 32-row group of an F2 weight's shard, or a piece of a parameter
//   whose gradient was reduce-scattered by NCCL into grad_shard):
//     wait (bounded, acquire) until the group's count reaches its expected arrivals,
//     g = own rows of the local fp32 gradient + the peers' inbox slots in rank order
//         (a fixed order: the result does not depend on arrival timing),
//     AdamATan2 + EMA on the fp32 master / state shards, bf16 copy into the shard that the
//     next step's F1 GEMMs (or the NCCL all-gather) read.
// All traffic here is local HBM; NVLink carried the gradient during the backward.
//
// Work item layout (int64 x 6): shard element begin, element count, offset of the rank's own
// rows in the full fp32 gradient (-1: the gradient is in grad_shard at `begin`), counter index
// (int32 elements from the symmetric buffer base; -1: no wait), expected count, and the index
// of the weight's first F2 region count in `ran` (-1: none). A weight whose F2 GEMM did not run
// this step (no gradient through it; every rank runs the same recurrence schedule, so no rank
// pushed) has that count at zero: its item neither waits nor reads the inbox, and its gradient
// is the rank's own rows, which are zero.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "collective_jobs.cuh"
#include "common.cuh"

namespace hrm {

at::Tensor device_error_word();  // errors.cu
CopyJobs decode_copy_jobs(const at::Tensor& d);  // gemm_tcgen05.cu

namespace {

struct ShardUpdateArgs {
  const long long* items;
  int n_items;
  const int* ran;      // local F2 region counts (zeroed at the start of every step)
  float* buf;          // this rank's fp32 symmetric buffer
  long master, m, v, ema, grad_shard, inbox, inbox_stride;  // fp32 element offsets into buf (m / ema: -1 = absent)
  const float* full_grad;
  __nv_bfloat16* shard16;
  int world, rank;
  const float* hyper;
  float beta1, beta2, wd, ema_decay;
  int* err;
};

__device__ __forceinline__ int ld_acquire_sys_s32(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void update4(const ShardUpdateArgs& a, long i, float4 g4, float lr, float ibc1, float ibc2) {
  float* P = a.buf + a.master + i;
  float* V = a.buf + a.v + i;
  float4 p4 = *reinterpret_cast<float4*>(P);
  float4 v4 = *reinterpret_cast<float4*>(V);
  float4 m4 = a.m >= 0 ? *reinterpret_cast<float4*>(a.buf + a.m + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  float* pp = &p4.x; float* vv = &v4.x; float* mm = &m4.x;
  const float* gg = &g4.x;
#pragma unroll
  for (int e = 0; e < 4; ++e)
    pp[e] = adam_atan2_update(pp[e], gg[e], a.m >= 0, mm[e], vv[e], lr, ibc1, ibc2, a.beta1, a.beta2, a.wd);
  *reinterpret_cast<float4*>(P) = p4;
  *reinterpret_cast<float4*>(V) = v4;
  if (a.m >= 0) *reinterpret_cast<float4*>(a.buf + a.m + i) = m4;
  if (a.ema >= 0) {
    float4 e4 = *reinterpret_cast<float4*>(a.buf + a.ema + i);
    const float d = 1.f - a.ema_decay;
    e4.x += d * (p4.x - e4.x); e4.y += d * (p4.y - e4.y); e4.z += d * (p4.z - e4.z); e4.w += d * (p4.w - e4.w);
    *reinterpret_cast<float4*>(a.buf + a.ema + i) = e4;
  }
  *reinterpret_cast<uint2*>(a.shard16 + i) = make_uint2(pack_bf16x2(p4.x, p4.y), pack_bf16x2(p4.z, p4.w));
}

__device__ __forceinline__ void update1(const ShardUpdateArgs& a, long i, float g, float lr, float ibc1, float ibc2) {
  float v = a.buf[a.v + i];
  float m = a.m >= 0 ? a.buf[a.m + i] : 0.f;
  const float p = adam_atan2_update(a.buf[a.master + i], g, a.m >= 0, m, v, lr, ibc1, ibc2, a.beta1,
                                    a.beta2, a.wd);
  a.buf[a.master + i] = p;
  a.buf[a.v + i] = v;
  if (a.m >= 0) a.buf[a.m + i] = m;
  if (a.ema >= 0) a.buf[a.ema + i] += (1.f - a.ema_decay) * (p - a.buf[a.ema + i]);
  a.shard16[i] = __float2bfloat16(p);
}

__global__ void __launch_bounds__(256) shard_update_kernel(const ShardUpdateArgs a) {
  __shared__ int ready;
  const float lr = a.hyper[0], ibc1 = a.hyper[1], ibc2 = a.hyper[2];
  for (int it = blockIdx.x; it < a.n_items; it += gridDim.x) {
    const long long* d = a.items + 6L * it;
    const long begin = d[0], own = d[2], ran_idx = d[5];
    const int count = (int)d[1], expected = (int)d[4];
    const long cnt = (ran_idx >= 0 && __ldcg(a.ran + ran_idx) == 0) ? -1 : d[3];
    if (cnt >= 0) {
      if (threadIdx.x == 0) {
        const int* c = reinterpret_cast<const int*>(a.buf) + cnt;
        const unsigned long long t0 = globaltimer_ns();
        int ok = 1;
        while (ld_acquire_sys_s32(c) < expected) {
          if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
            report_error(a.err, kErrPeerWaitTimeout, 7);
            ok = 0;
            break;
          }
          __nanosleep(256);
        }
        ready = ok;
      }
      __syncthreads();
      const int ok = ready;
      __syncthreads();  // `ready` is rewritten by the next item's wait
      if (!ok) continue;
    }
    const float* gsrc = own >= 0 ? a.full_grad + own : a.buf + a.grad_shard + begin;
    const bool inbox = cnt >= 0;
    const int n4 = count >> 2;
    for (int q = threadIdx.x; q < n4; q += blockDim.x) {
      float4 g4 = __ldcg(reinterpret_cast<const float4*>(gsrc) + q);
      if (inbox) {
        for (int src = 0; src < a.world; ++src) {
          if (src == a.rank) continue;
          const float4 t = __ldcg(reinterpret_cast<const float4*>(a.buf + a.inbox + (long)src * a.inbox_stride + begin) + q);
          g4.x += t.x; g4.y += t.y; g4.z += t.z; g4.w += t.w;
        }
      }
      update4(a, begin + 4L * q, g4, lr, ibc1, ibc2);
    }
    for (int e = 4 * n4 + threadIdx.x; e < count; e += blockDim.x) {
      float g = __ldcg(gsrc + e);
      if (inbox)
        for (int src = 0; src < a.world; ++src)
          if (src != a.rank) g += __ldcg(a.buf + a.inbox + (long)src * a.inbox_stride + begin + e);
      update1(a, begin + e, g, lr, ibc1, ibc2);
    }
  }
}

// Copy jobs with no GEMM to ride on (the first weight of a step, the pushes left at the end of
// the backward): 8 warps per CTA, one CTA per SM.
__global__ void __launch_bounds__(256) copy_jobs_kernel(const CopyJobs j) {
  run_copy_jobs(j, (int)(blockIdx.x * 8 + (threadIdx.x >> 5)), (int)(gridDim.x * 8), (int)(threadIdx.x & 31));
}

}  // namespace

void copy_jobs(const at::Tensor& jobs, int64_t device) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  const CopyJobs j = decode_copy_jobs(jobs);
  if (j.g_src == nullptr && j.p_src == nullptr) return;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, (int)device);
  copy_jobs_kernel<<<sms, 256, 0, at::cuda::getCurrentCUDAStream()>>>(j);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// items: device int64 [n, 6] (see the file header); buf: this rank's fp32 symmetric buffer;
// offs: fp32 element offsets {master, exp_avg (-1), exp_avg_sq, param_ema (-1), grad_shard,
// inbox, inbox_stride}; full_grad: the local fp32 gradient of all parameters; shard16: this
// rank's bf16 shard buffer (same element indexing as the fp32 shard regions); ran: the local
// F2 region counts.
void shard_update(const at::Tensor& items, const at::Tensor& buf, const std::vector<int64_t>& offs,
                  const at::Tensor& full_grad, const at::Tensor& shard16, const at::Tensor& ran, int64_t world,
                  int64_t rank, const at::Tensor& hyper, double beta1, double beta2, double wd, double ema_decay) {
  TORCH_CHECK(items.is_cuda() && items.scalar_type() == at::kLong && items.dim() == 2 && items.size(1) == 6,
              "shard_update: items must be CUDA int64 [n, 6]");
  TORCH_CHECK(buf.is_cuda() && buf.scalar_type() == at::kFloat && full_grad.scalar_type() == at::kFloat,
              "shard_update: fp32 buffers expected");
  TORCH_CHECK(shard16.scalar_type() == at::kBFloat16 && offs.size() == 7, "shard_update: bad arguments");
  for (int i = 0; i < 7; ++i)
    TORCH_CHECK(offs[i] < 0 || offs[i] % 4 == 0, "shard_update: region offsets must be 16-byte aligned");
  c10::cuda::CUDAGuard guard(buf.device());
  ShardUpdateArgs a{};
  a.items = reinterpret_cast<const long long*>(items.data_ptr<int64_t>());
  a.n_items = (int)items.size(0);
  TORCH_CHECK(ran.is_cuda() && ran.scalar_type() == at::kInt, "shard_update: ran must be CUDA int32");
  a.ran = ran.data_ptr<int>();
  a.buf = buf.data_ptr<float>();
  a.master = offs[0]; a.m = offs[1]; a.v = offs[2]; a.ema = offs[3];
  a.grad_shard = offs[4]; a.inbox = offs[5]; a.inbox_stride = offs[6];
  a.full_grad = full_grad.data_ptr<float>();
  a.shard16 = reinterpret_cast<__nv_bfloat16*>(shard16.data_ptr());
  a.world = (int)world; a.rank = (int)rank;
  a.hyper = hyper.data_ptr<float>();
  a.beta1 = (float)beta1; a.beta2 = (float)beta2; a.wd = (float)wd; a.ema_decay = (float)ema_decay;
  a.err = device_error_word().data_ptr<int>();
  if (a.n_items == 0) return;
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, buf.get_device());
  const int grid = std::min(a.n_items, sms * 8);
  shard_update_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace hrm
