// Cross-entropy over a chunk of bf16 logits, fused with its gradient (sm_100a).
//
// One CTA per row: pass 1 computes max and sum(exp) online, pass 2 overwrites
// the logits with d(loss)/d(logits) = (softmax - onehot) * grad_scale in
// place.  The row stays in L2 between the passes.  Used by the chunked fused
// linear cross-entropy: the lm-head GEMM writes a logits chunk, this kernel
// turns it into its gradient, and the two backward GEMMs consume it, so the
// full [tokens, vocab] logits never exist.
//
// Reference parity: chunked / fused linear cross-entropy of
// veomni/ops/kernels/cross_entropy/ (chunk_loss, liger fused linear CE).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace pm {

__global__ void __launch_bounds__(512) ce_fwd_bwd_kernel(__nv_bfloat16* __restrict__ logits, int V, long long ld,
                                                         const long long* __restrict__ labels, int ignore_index,
                                                         float grad_scale, float* __restrict__ loss_sum,
                                                         float* __restrict__ row_loss) {
  __shared__ float s_m[16], s_s[16];
  const int row = blockIdx.x;
  __nv_bfloat16* z = logits + (size_t)row * ld;
  long long lab = labels[row];
  bool ignore = lab == ignore_index;
  if (!ignore && (lab < 0 || lab >= V)) {  // out-of-vocabulary label: record and treat as ignored
    if (threadIdx.x == 0) set_error(kErrBounds);
    ignore = true;
    lab = 0;
  }
  float m = -INFINITY, s = 0.f;
  const int V2 = V / 2;
  const __nv_bfloat162* z2 = reinterpret_cast<const __nv_bfloat162*>(z);
  for (int i = threadIdx.x; i < V2; i += blockDim.x) {
    const __nv_bfloat162 p = z2[i];
    const float a = __low2float(p), b = __high2float(p);
    const float nm = fmaxf(m, fmaxf(a, b));
    s = s * __expf(m - nm) + __expf(a - nm) + __expf(b - nm);
    m = nm;
  }
  if ((V & 1) && threadIdx.x == 0) {
    const float a = __bfloat162float(z[V - 1]);
    const float nm = fmaxf(m, a);
    s = s * __expf(m - nm) + __expf(a - nm);
    m = nm;
  }
  // warp then block combine of (m, s)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float os = __shfl_xor_sync(0xffffffffu, s, o);
    const float nm = fmaxf(m, om);
    s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
    m = nm;
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { s_m[w] = m; s_s[w] = s; }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    m = lane < nw ? s_m[lane] : -INFINITY;
    s = lane < nw ? s_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, m, o);
      const float os = __shfl_xor_sync(0xffffffffu, s, o);
      const float nm = fmaxf(m, om);
      s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
      m = nm;
    }
    if (lane == 0) { s_m[0] = m; s_s[0] = s; }
  }
  __syncthreads();
  const float lse = s_m[0] + logf(s_s[0]);
  if (threadIdx.x == 0) {
    const float l = ignore ? 0.f : lse - __bfloat162float(z[lab]);
    if (row_loss) row_loss[row] = l;
    if (!ignore) atomicAdd(loss_sum, l);
  }
  __syncthreads();  // z[lab] read before it is overwritten
  const float gsc = ignore ? 0.f : grad_scale;
  __nv_bfloat162* w2 = reinterpret_cast<__nv_bfloat162*>(z);
  for (int i = threadIdx.x; i < V2; i += blockDim.x) {
    const __nv_bfloat162 p = w2[i];
    float a = __expf(__low2float(p) - lse), b = __expf(__high2float(p) - lse);
    if (2 * i == lab) a -= 1.f;
    if (2 * i + 1 == lab) b -= 1.f;
    w2[i] = __floats2bfloat162_rn(a * gsc, b * gsc);
  }
  if ((V & 1) && threadIdx.x == 0) {
    float a = __expf(__bfloat162float(z[V - 1]) - lse);
    if (V - 1 == lab) a -= 1.f;
    z[V - 1] = __float2bfloat16(a * gsc);
  }
}

// logits: [n, V] bf16 (overwritten with the gradient); labels: [n] int64.
// Adds the summed loss of non-ignored rows to loss_sum (fp32 scalar).
void ce_fwd_bwd(torch::Tensor logits, torch::Tensor labels, int64_t ignore_index, double grad_scale,
                torch::Tensor loss_sum, c10::optional<torch::Tensor> row_loss) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == torch::kBFloat16 && logits.stride(-1) == 1, "logits bf16");
  TORCH_CHECK(logits.stride(0) % 2 == 0, "row stride must be even");
  TORCH_CHECK(labels.scalar_type() == torch::kInt64 && labels.is_contiguous(), "labels int64");
  PM_CHECK_CUDA(labels); PM_CHECK_CUDA(loss_sum); PM_CHECK_CUDA_OPT(row_loss);
  TORCH_CHECK(labels.numel() == logits.size(0), "one label per row");
  const int n = (int)logits.size(0);
  const int V = (int)logits.size(1);
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(logits.device());
  ce_fwd_bwd_kernel<<<n, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
      (__nv_bfloat16*)logits.data_ptr(), V, logits.stride(0), reinterpret_cast<const long long*>(labels.data_ptr<int64_t>()), (int)ignore_index,
      (float)grad_scale, loss_sum.data_ptr<float>(), row_loss.has_value() ? row_loss->data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace pm

PM_DEFINE_ERROR_QUERY(pm_error_loss)
