// Multi-tensor fused AdamW and squared-L2-norm kernels (sm_100a).
//
// One launch updates every parameter tensor of a group: a device table of
// per-tensor pointers plus a chunk table (tensor index, start) lets a single
// grid walk all chunks.  fp32 master weights, fp32 moments, fp32 or bf16
// gradients; optionally writes a bf16 copy of the updated weights (the
// compute copy the expert GEMMs read), so no separate cast pass is needed.
//
// sq_norm: per-tensor weighted sum of squares for gradient clipping.  Each
// table entry carries a weight, which is how redundant expert copies are
// excluded from the norm (each logical expert is counted once).
//
// Reference parity: fused torch AdamW (veomni/optim/optimizer.py:261-330) and
// veomni_clip_grad_norm with redundant-slot masks
// (veomni/distributed/fsdp2/clip_grad_norm.py:94-176,
// veomni/distributed/moe/hiermoe/expert_swap.py:7254-7266).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace pm {

struct AdamTensor {
  float* p;
  const void* g;
  float* m;
  float* v;
  __nv_bfloat16* shadow;  // optional bf16 copy of p
  long long n;
  int g_bf16;
  int pad;
};

constexpr int kChunk = 1 << 16;

__global__ void __launch_bounds__(256) adamw_kernel(const AdamTensor* __restrict__ tensors,
                                                    const int2* __restrict__ chunks, int nchunks, float lr, float beta1,
                                                    float beta2, float eps, float wd, float bc1, float bc2,
                                                    const float* __restrict__ grad_scale) {
  const float gs = grad_scale ? *grad_scale : 1.f;
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const int2 ch = chunks[c];
    const AdamTensor t = tensors[ch.x];
    const long long beg = (long long)ch.y * kChunk;
    const long long end = min(beg + (long long)kChunk, t.n);
    // vectorized body (4 elements / thread / iteration); the tail is scalar
    const long long vend = beg + ((end - beg) & ~3LL);
    for (long long i = beg + threadIdx.x * 4; i < vend; i += blockDim.x * 4) {
      float4 p = *reinterpret_cast<float4*>(t.p + i);
      float4 m = *reinterpret_cast<float4*>(t.m + i);
      float4 v = *reinterpret_cast<float4*>(t.v + i);
      float g[4];
      if (t.g_bf16) {
        const uint2 q = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(t.g) + i);
        g[0] = bf16_lo(q.x); g[1] = bf16_hi(q.x); g[2] = bf16_lo(q.y); g[3] = bf16_hi(q.y);
      } else {
        const float4 q = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(t.g) + i);
        g[0] = q.x; g[1] = q.y; g[2] = q.z; g[3] = q.w;
      }
      float* pp = &p.x;
      float* mm = &m.x;
      float* vv = &v.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float gj = g[j] * gs;
        mm[j] = beta1 * mm[j] + (1.f - beta1) * gj;
        vv[j] = beta2 * vv[j] + (1.f - beta2) * gj * gj;
        const float denom = sqrtf(vv[j] / bc2) + eps;
        pp[j] = pp[j] * (1.f - lr * wd) - lr * (mm[j] / bc1) / denom;
      }
      *reinterpret_cast<float4*>(t.p + i) = p;
      *reinterpret_cast<float4*>(t.m + i) = m;
      *reinterpret_cast<float4*>(t.v + i) = v;
      if (t.shadow)
        *reinterpret_cast<uint2*>(t.shadow + i) = make_uint2(pack_bf16(p.x, p.y), pack_bf16(p.z, p.w));
    }
    for (long long i = vend + threadIdx.x; i < end; i += blockDim.x) {
      const float gj = (t.g_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(t.g)[i])
                                 : reinterpret_cast<const float*>(t.g)[i]) * gs;
      const float m = beta1 * t.m[i] + (1.f - beta1) * gj;
      const float v = beta2 * t.v[i] + (1.f - beta2) * gj * gj;
      t.m[i] = m;
      t.v[i] = v;
      const float p = t.p[i] * (1.f - lr * wd) - lr * (m / bc1) / (sqrtf(v / bc2) + eps);
      t.p[i] = p;
      if (t.shadow) t.shadow[i] = __float2bfloat16(p);
    }
  }
}

struct NormTensor {
  const void* g;
  long long n;
  float weight;
  int g_bf16;
};

__global__ void __launch_bounds__(256) sq_norm_kernel(const NormTensor* __restrict__ tensors,
                                                      const int2* __restrict__ chunks, int nchunks,
                                                      float* __restrict__ out) {
  __shared__ float red[8];
  float acc = 0.f;
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const int2 ch = chunks[c];
    const NormTensor t = tensors[ch.x];
    const long long beg = (long long)ch.y * kChunk;
    const long long end = min(beg + (long long)kChunk, t.n);
    float part = 0.f;
    if (t.g_bf16) {
      const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(t.g);
      const bool vec_ok = (reinterpret_cast<uintptr_t>(g + beg) & 15) == 0;
      const long long vend = vec_ok ? beg + ((end - beg) & ~7LL) : beg;
      for (long long i = beg + threadIdx.x * 8; i < vend; i += blockDim.x * 8) {
        const uint4 q = *reinterpret_cast<const uint4*>(g + i);
        const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float a = bf16_lo(u[j]), b = bf16_hi(u[j]);
          part += a * a + b * b;
        }
      }
      for (long long i = vend + threadIdx.x; i < end; i += blockDim.x) {
        const float x = __bfloat162float(g[i]);
        part += x * x;
      }
    } else {
      const float* g = reinterpret_cast<const float*>(t.g);
      const bool vec_ok = (reinterpret_cast<uintptr_t>(g + beg) & 15) == 0;
      const long long vend = vec_ok ? beg + ((end - beg) & ~3LL) : beg;
      for (long long i = beg + threadIdx.x * 4; i < vend; i += blockDim.x * 4) {
        const float4 v = *reinterpret_cast<const float4*>(g + i);
        part += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
      for (long long i = vend + threadIdx.x; i < end; i += blockDim.x) part += g[i] * g[i];
    }
    acc += part * t.weight;
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < 8 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) atomicAdd(out, v);
  }
}

static int sms_opt() {
  int dev, n;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

// The host-side tables are packed into one int64 CPU tensor by the caller-facing
// helpers below and uploaded once per call.
static torch::Tensor upload(const void* data, size_t bytes, const torch::Device& dev) {
  auto cpu = torch::empty({(int64_t)((bytes + 7) / 8)}, torch::TensorOptions().dtype(torch::kInt64).pinned_memory(true));
  memcpy(cpu.data_ptr(), data, bytes);
  return cpu.to(dev, /*non_blocking=*/true);
}

// Tables are cached by the Python caller: build_adam_table returns a device
// tensor holding [AdamTensor...][int2 chunks...] and the chunk count.
std::vector<torch::Tensor> adamw_build_table(std::vector<torch::Tensor> params, std::vector<torch::Tensor> grads,
                                             std::vector<torch::Tensor> exp_avg, std::vector<torch::Tensor> exp_avg_sq,
                                             std::vector<c10::optional<torch::Tensor>> shadows) {
  const size_t nt = params.size();
  TORCH_CHECK(grads.size() == nt && exp_avg.size() == nt && exp_avg_sq.size() == nt && shadows.size() == nt,
              "table lengths differ");
  std::vector<AdamTensor> ts(nt);
  std::vector<int2> chunks;
  for (size_t i = 0; i < nt; ++i) {
    auto& p = params[i];
    TORCH_CHECK(p.is_cuda() && p.scalar_type() == torch::kFloat32 && p.is_contiguous(), "params must be fp32");
    TORCH_CHECK(grads[i].is_contiguous() && grads[i].numel() == p.numel(), "grad shape");
    TORCH_CHECK(grads[i].is_cuda() && exp_avg[i].is_cuda() && exp_avg_sq[i].is_cuda(), "AdamW tensors must be CUDA");
    TORCH_CHECK(!shadows[i].has_value() || (shadows[i]->is_cuda() && shadows[i]->numel() == p.numel() &&
                                            shadows[i]->scalar_type() == torch::kBFloat16), "bf16 shadow");
    TORCH_CHECK(exp_avg[i].numel() == p.numel() && exp_avg_sq[i].numel() == p.numel(), "moment shape");
    TORCH_CHECK(grads[i].scalar_type() == torch::kFloat32 || grads[i].scalar_type() == torch::kBFloat16, "grad dtype");
    ts[i].p = p.data_ptr<float>();
    ts[i].g = grads[i].data_ptr();
    ts[i].m = exp_avg[i].data_ptr<float>();
    ts[i].v = exp_avg_sq[i].data_ptr<float>();
    ts[i].shadow = shadows[i].has_value() ? (__nv_bfloat16*)shadows[i]->data_ptr() : nullptr;
    ts[i].n = p.numel();
    ts[i].g_bf16 = grads[i].scalar_type() == torch::kBFloat16;
    TORCH_CHECK((reinterpret_cast<uintptr_t>(ts[i].p) & 15) == 0 && (reinterpret_cast<uintptr_t>(ts[i].m) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(ts[i].v) & 15) == 0,
                "AdamW tensors must be 16-byte aligned");
    const long long nch = (p.numel() + kChunk - 1) / kChunk;
    for (long long c = 0; c < nch; ++c) chunks.push_back(make_int2((int)i, (int)c));
  }
  const size_t tb = nt * sizeof(AdamTensor);
  std::vector<uint8_t> blob(tb + chunks.size() * sizeof(int2));
  memcpy(blob.data(), ts.data(), tb);
  memcpy(blob.data() + tb, chunks.data(), chunks.size() * sizeof(int2));
  auto dev = params.empty() ? torch::Device(torch::kCUDA) : params[0].device();
  auto table = upload(blob.data(), blob.size(), dev);
  auto meta = torch::tensor({(int64_t)nt, (int64_t)chunks.size()}, torch::kInt64);
  return {table, meta};
}

void adamw_step(torch::Tensor table, torch::Tensor meta, double lr, double beta1, double beta2, double eps, double wd,
                int64_t step, c10::optional<torch::Tensor> grad_scale) {
  PM_CHECK_CUDA(table);
  PM_CHECK_CUDA_OPT(grad_scale);
  const int64_t nt = meta[0].item<int64_t>();
  const int nchunks = (int)meta[1].item<int64_t>();
  if (nchunks == 0) return;
  c10::cuda::CUDAGuard guard(table.device());
  const AdamTensor* tp = reinterpret_cast<const AdamTensor*>(table.data_ptr());
  const int2* cp = reinterpret_cast<const int2*>(reinterpret_cast<const uint8_t*>(table.data_ptr()) + nt * sizeof(AdamTensor));
  const float bc1 = 1.f - (float)std::pow(beta1, (double)step);
  const float bc2 = 1.f - (float)std::pow(beta2, (double)step);
  const float* gs = grad_scale.has_value() ? grad_scale->data_ptr<float>() : nullptr;
  const int grid = std::min(nchunks, sms_opt() * 8);
  adamw_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(tp, cp, nchunks, (float)lr, (float)beta1,
                                                                   (float)beta2, (float)eps, (float)wd, bc1, bc2, gs);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

std::vector<torch::Tensor> sq_norm_build_table(std::vector<torch::Tensor> grads, std::vector<double> weights) {
  TORCH_CHECK(grads.size() == weights.size(), "weights");
  std::vector<NormTensor> ts(grads.size());
  std::vector<int2> chunks;
  for (size_t i = 0; i < grads.size(); ++i) {
    TORCH_CHECK(grads[i].is_contiguous() && grads[i].is_cuda(), "grads must be contiguous CUDA tensors");
    ts[i].g = grads[i].data_ptr();
    ts[i].n = grads[i].numel();
    ts[i].weight = (float)weights[i];
    ts[i].g_bf16 = grads[i].scalar_type() == torch::kBFloat16;
    TORCH_CHECK(ts[i].g_bf16 || grads[i].scalar_type() == torch::kFloat32, "grad dtype");
    const long long nch = (grads[i].numel() + kChunk - 1) / kChunk;
    for (long long c = 0; c < nch; ++c) chunks.push_back(make_int2((int)i, (int)c));
  }
  const size_t tb = ts.size() * sizeof(NormTensor);
  std::vector<uint8_t> blob(tb + chunks.size() * sizeof(int2) + 8);
  memcpy(blob.data(), ts.data(), tb);
  memcpy(blob.data() + tb, chunks.data(), chunks.size() * sizeof(int2));
  auto dev = grads.empty() ? torch::Device(torch::kCUDA) : grads[0].device();
  auto table = upload(blob.data(), blob.size(), dev);
  auto meta = torch::tensor({(int64_t)ts.size(), (int64_t)chunks.size()}, torch::kInt64);
  return {table, meta};
}

// out (fp32 scalar tensor) += sum_i weight_i * ||g_i||^2
void sq_norm(torch::Tensor table, torch::Tensor meta, torch::Tensor out) {
  PM_CHECK_CUDA(table);
  PM_CHECK_CUDA(out);
  const int64_t nt = meta[0].item<int64_t>();
  const int nchunks = (int)meta[1].item<int64_t>();
  if (nchunks == 0) return;
  c10::cuda::CUDAGuard guard(table.device());
  const NormTensor* tp = reinterpret_cast<const NormTensor*>(table.data_ptr());
  const int2* cp = reinterpret_cast<const int2*>(reinterpret_cast<const uint8_t*>(table.data_ptr()) + nt * sizeof(NormTensor));
  const int grid = std::min(nchunks, sms_opt() * 8);
  sq_norm_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(tp, cp, nchunks, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace pm

PM_DEFINE_ERROR_QUERY(pm_error_optim)
