// MoE routing kernels (sm_100a): router softmax/top-k, the deterministic
// expert-contiguous dispatch plan, row gather and weighted-sum combine.
//
// router_topk_fwd: one warp per token.  logits(+bias) -> fp32 softmax ->
//   top-k (ties resolved to the lower expert id) -> optional renormalisation.
//   Logical->physical remapping through the placement LUT happens in the
//   dispatch plan, so the logical top-k is kept bit-for-bit.
// router_topk_bwd: recomputes the softmax and returns d(logits) for the
//   routing-weight gradient plus the load-balancing loss gradient.
// moe_plan: counting sort of the (token, k) assignments by physical slot with
//   a stable (token-major) order; segments padded to multiples of 128 rows so
//   each GEMM tile belongs to one expert.  No host synchronisation.
//
// Reference parity: Qwen3MoeTopKRouter
// (veomni/models/transformers/qwen3_moe/generated/patched_modeling_qwen3_moe_gpu.py:306-337),
// the permute/unpermute helpers of veomni/ops/kernels/moe/_kernels/kernel/moe.py:29-418,
// map_logical_to_physical (veomni/distributed/moe/hiermoe/expert_swap.py:5903-5935)
// and the load-balancing loss of veomni/ops/kernels/load_balancing_loss/triton.py:37-354.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace pm {

constexpr int kMaxE = 512;

// EPL = experts per lane (E / 32, E <= 512)
template <int EPL>
__global__ void __launch_bounds__(256) router_topk_fwd_kernel(const float* __restrict__ logits,
                                                              const float* __restrict__ bias, int T, int E, int K,
                                                              bool renorm, int* __restrict__ idx,
                                                              float* __restrict__ wts, float* __restrict__ prob_sum,
                                                              float* __restrict__ count) {
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  __shared__ float s_prob[kMaxE];
  __shared__ float s_cnt[kMaxE];
  for (int i = threadIdx.x; i < E; i += blockDim.x) { s_prob[i] = 0.f; s_cnt[i] = 0.f; }
  __syncthreads();
  if (t < T) {
    float z[EPL];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      const int e = j * 32 + lane;
      z[j] = e < E ? logits[(size_t)t * E + e] + (bias ? bias[e] : 0.f) : -INFINITY;
      mx = fmaxf(mx, z[j]);
    }
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      z[j] = (j * 32 + lane) < E ? __expf(z[j] - mx) : 0.f;
      sum += z[j];
    }
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      z[j] *= inv;
      if (j * 32 + lane < E) atomicAdd(&s_prob[j * 32 + lane], z[j]);
    }
    // top-k by repeated warp argmax
    float selw = 0.f, tot = 0.f;
    int sele = 0;
    bool taken[EPL];
#pragma unroll
    for (int j = 0; j < EPL; ++j) taken[j] = false;
    for (int kk = 0; kk < K; ++kk) {
      float best = -1.f;
      int be = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < EPL; ++j) {
        const int e = j * 32 + lane;
        if (e < E && !taken[j] && (z[j] > best)) { best = z[j]; be = e; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oe = __shfl_xor_sync(0xffffffffu, be, o);
        if (ob > best || (ob == best && oe < be)) { best = ob; be = oe; }
      }
      if ((be & 31) == lane) taken[be >> 5] = true;
      if (lane == kk) { selw = best; sele = be; }
      tot += best;
    }
    if (lane < K) {
      idx[(size_t)t * K + lane] = sele;
      wts[(size_t)t * K + lane] = renorm ? selw / tot : selw;
      atomicAdd(&s_cnt[sele], 1.f);
    }
  }
  __syncthreads();
  if (prob_sum)
    for (int i = threadIdx.x; i < E; i += blockDim.x) {
      atomicAdd(&prob_sum[i], s_prob[i]);
      atomicAdd(&count[i], s_cnt[i]);
    }
}

// d(logits) = p * (g - <g, p>), g_e = aux_coef[e] + (routing-weight grad of e if selected)
template <int EPL>
__global__ void __launch_bounds__(256) router_topk_bwd_kernel(const float* __restrict__ logits,
                                                              const float* __restrict__ bias, const int* __restrict__ idx,
                                                              const float* __restrict__ dw, const float* __restrict__ aux,
                                                              int T, int E, int K, bool renorm,
                                                              __nv_bfloat16* __restrict__ dlogits) {
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float z[EPL];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = j * 32 + lane;
    z[j] = e < E ? logits[(size_t)t * E + e] + (bias ? bias[e] : 0.f) : -INFINITY;
    mx = fmaxf(mx, z[j]);
  }
  mx = warp_max(mx);
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    z[j] = (j * 32 + lane) < E ? __expf(z[j] - mx) : 0.f;
    sum += z[j];
  }
  sum = warp_sum(sum);
  const float inv = 1.f / sum;
#pragma unroll
  for (int j = 0; j < EPL; ++j) z[j] *= inv;
  // selected experts' probabilities and the renormalisation terms
  float my_dw = 0.f, my_p = 0.f;
  int my_e = -1;
  if (lane < K) {
    my_e = idx[(size_t)t * K + lane];
    my_dw = dw[(size_t)t * K + lane];
  }
  // gather p for the selected experts (E/32 registers per lane -> explicit select)
  float p_sel = 0.f;
  for (int kk = 0; kk < K; ++kk) {
    const int e = __shfl_sync(0xffffffffu, my_e, kk);
    float val = 0.f;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      const float cand = __shfl_sync(0xffffffffu, z[j], e & 31);
      if ((e >> 5) == j) val = cand;
    }
    if (lane == kk) p_sel = val;
  }
  my_p = p_sel;
  float S = warp_sum(lane < K ? my_p : 0.f);
  float gsel = my_dw;  // d/dp of the selected expert
  if (renorm) {
    const float wsel = my_p / S;
    const float c = warp_sum(lane < K ? my_dw * wsel : 0.f);
    gsel = (my_dw - c) / S;
  }
  float g[EPL];
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = j * 32 + lane;
    g[j] = (aux && e < E) ? aux[e] : 0.f;
  }
  for (int kk = 0; kk < K; ++kk) {
    const int e = __shfl_sync(0xffffffffu, my_e, kk);
    const float ge = __shfl_sync(0xffffffffu, gsel, kk);
    if ((e & 31) == lane) {
#pragma unroll
      for (int j = 0; j < EPL; ++j)
        if ((e >> 5) == j) g[j] += ge;
    }
  }
  float dot = 0.f;
#pragma unroll
  for (int j = 0; j < EPL; ++j) dot += g[j] * z[j];
  dot = warp_sum(dot);
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = j * 32 + lane;
    if (e < E) dlogits[(size_t)t * E + e] = __float2bfloat16(z[j] * (g[j] - dot));
  }
}

#define PM_EPL_DISPATCH(E, ...)                                        \
  if ((E) <= 32) { constexpr int EPL = 1; __VA_ARGS__; }                \
  else if ((E) <= 64) { constexpr int EPL = 2; __VA_ARGS__; }           \
  else if ((E) <= 128) { constexpr int EPL = 4; __VA_ARGS__; }          \
  else if ((E) <= 256) { constexpr int EPL = 8; __VA_ARGS__; }          \
  else { constexpr int EPL = 16; __VA_ARGS__; }

// Returns idx [T,K] int32, weights [T,K] fp32, prob_sum [E], count [E].
std::vector<torch::Tensor> router_topk_fwd(torch::Tensor logits, c10::optional<torch::Tensor> bias, int64_t K,
                                           bool renorm) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == torch::kFloat32 && logits.is_contiguous(), "logits fp32");
  PM_CHECK_CUDA_OPT(bias);
  if (bias.has_value()) TORCH_CHECK(bias->scalar_type() == torch::kFloat32 && bias->numel() == logits.size(-1), "bias");
  const int E = (int)logits.size(-1);
  const int T = (int)(logits.numel() / E);
  TORCH_CHECK(E <= kMaxE && K <= 32 && K <= E, "router supports E <= 512, K <= 32");
  c10::cuda::CUDAGuard guard(logits.device());
  auto opt = logits.options();
  auto idx = torch::empty({T, K}, opt.dtype(torch::kInt32));
  auto w = torch::empty({T, K}, opt);
  auto ps = torch::zeros({E}, opt);
  auto cnt = torch::zeros({E}, opt);
  if (T == 0) return {idx, w, ps, cnt};
  const float* bp = bias.has_value() ? bias->data_ptr<float>() : nullptr;
  auto stream = at::cuda::getCurrentCUDAStream();
  PM_EPL_DISPATCH(E, router_topk_fwd_kernel<EPL><<<(T + 7) / 8, 256, 0, stream>>>(
                         logits.data_ptr<float>(), bp, T, E, (int)K, renorm, idx.data_ptr<int>(), w.data_ptr<float>(),
                         ps.data_ptr<float>(), cnt.data_ptr<float>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {idx, w, ps, cnt};
}

torch::Tensor router_topk_bwd(torch::Tensor logits, c10::optional<torch::Tensor> bias, torch::Tensor idx,
                              torch::Tensor dw, c10::optional<torch::Tensor> aux, bool renorm) {
  const int E = (int)logits.size(-1);
  const int T = (int)(logits.numel() / E);
  const int K = (int)idx.size(-1);
  TORCH_CHECK(dw.scalar_type() == torch::kFloat32 && dw.is_contiguous(), "dw fp32");
  PM_CHECK_CUDA(logits); PM_CHECK_CUDA(idx); PM_CHECK_CUDA(dw); PM_CHECK_CUDA_OPT(bias); PM_CHECK_CUDA_OPT(aux);
  c10::cuda::CUDAGuard guard(logits.device());
  auto dl = torch::empty({T, E}, logits.options().dtype(torch::kBFloat16));
  if (T == 0) return dl;
  const float* bp = bias.has_value() ? bias->data_ptr<float>() : nullptr;
  const float* ap = aux.has_value() ? aux->data_ptr<float>() : nullptr;
  auto stream = at::cuda::getCurrentCUDAStream();
  PM_EPL_DISPATCH(E, router_topk_bwd_kernel<EPL><<<(T + 7) / 8, 256, 0, stream>>>(
                         logits.data_ptr<float>(), bp, idx.data_ptr<int>(), dw.data_ptr<float>(), ap, T, E, K, renorm,
                         (__nv_bfloat16*)dl.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dl;
}

// ----------------------------------------------------------------------------
// Dispatch plan: counting sort by slot, stable in (token, k) order.
// ----------------------------------------------------------------------------
constexpr int kPlanChunk = 2048;  // assignments per CTA
constexpr int kPlanWarps = 8;

// slot_of(a) = lut[idx[a]]; slots outside [0, num_slots) are not local (skipped).
__global__ void __launch_bounds__(256) plan_count_kernel(const int* __restrict__ idx, const int* __restrict__ lut, int n,
                                                         int num_slots, int* __restrict__ block_counts) {
  extern __shared__ int hist[];
  for (int i = threadIdx.x; i < num_slots; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int beg = blockIdx.x * kPlanChunk;
  const int end = min(beg + kPlanChunk, n);
  for (int a = beg + threadIdx.x; a < end; a += blockDim.x) {
    const int s = lut ? lut[idx[a]] : idx[a];
    if (s >= 0 && s < num_slots) atomicAdd(&hist[s], 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < num_slots; i += blockDim.x) block_counts[(size_t)blockIdx.x * num_slots + i] = hist[i];
}

// One CTA: per-slot prefix over blocks, then padded exclusive scan over slots.
__global__ void __launch_bounds__(1024) plan_scan_kernel(int* __restrict__ block_counts, int nblocks, int num_slots,
                                                         int align, int* __restrict__ offsets, int* __restrict__ counts) {
  __shared__ int padded[1024];
  const int s = threadIdx.x;
  int total = 0;
  if (s < num_slots) {
    for (int b = 0; b < nblocks; ++b) {
      int* p = &block_counts[(size_t)b * num_slots + s];
      const int c = *p;
      *p = total;  // becomes the block's base within the slot
      total += c;
    }
    counts[s] = total;
    padded[s] = (total + align - 1) / align * align;
  }
  __syncthreads();
  if (s == 0) {
    int run = 0;
    for (int i = 0; i < num_slots; ++i) {
      offsets[i] = run;
      run += padded[i];
    }
    offsets[num_slots] = run;
  }
}

__global__ void __launch_bounds__(256) plan_scatter_kernel(const int* __restrict__ idx, const int* __restrict__ lut,
                                                           const float* __restrict__ w, int n, int K, int num_slots,
                                                           const int* __restrict__ block_base,
                                                           const int* __restrict__ offsets, int* __restrict__ row_of,
                                                           int* __restrict__ row_token, float* __restrict__ row_scale) {
  extern __shared__ int wbase[];  // [kPlanWarps][num_slots]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kPlanWarps * num_slots; i += blockDim.x) wbase[i] = 0;
  __syncthreads();
  const int beg = blockIdx.x * kPlanChunk;
  const int per_warp = kPlanChunk / kPlanWarps;
  const int wbeg = beg + warp * per_warp;
  const int wend = min(wbeg + per_warp, n);
  int* my = wbase + warp * num_slots;
  for (int a = wbeg + lane; a < wend; a += 32) {
    const int s = lut ? lut[idx[a]] : idx[a];
    if (s >= 0 && s < num_slots) atomicAdd(&my[s], 1);
  }
  __syncthreads();
  // exclusive prefix over warps + the block base
  for (int s = threadIdx.x; s < num_slots; s += blockDim.x) {
    int run = block_base[(size_t)blockIdx.x * num_slots + s] + offsets[s];
    for (int k = 0; k < kPlanWarps; ++k) {
      const int c = wbase[k * num_slots + s];
      wbase[k * num_slots + s] = run;
      run += c;
    }
  }
  __syncthreads();
  for (int a0 = wbeg; a0 < wend; a0 += 32) {
    const int a = a0 + lane;
    int s = -1;
    if (a < wend) s = lut ? lut[idx[a]] : idx[a];
    const bool local = s >= 0 && s < num_slots;
    const unsigned peers = __match_any_sync(0xffffffffu, local ? s : -1);
    const int rank = __popc(peers & ((1u << lane) - 1));
    int row = -1;
    if (local) row = my[s] + rank;
    __syncwarp();
    if (local && rank == 0) my[s] += __popc(peers);
    __syncwarp();
    if (a < wend) {
      row_of[a] = row;
      if (local) {
        row_token[row] = a / K;
        row_scale[row] = w ? w[a] : 1.f;
      }
    }
  }
}

// Padding rows of every slot segment: token -1, scale 0.
__global__ void plan_pad_kernel(const int* __restrict__ offsets, const int* __restrict__ counts, int num_slots,
                                int* __restrict__ row_token, float* __restrict__ row_scale) {
  const int s = blockIdx.x;
  const int beg = offsets[s] + counts[s], end = offsets[s + 1];
  for (int r = beg + threadIdx.x; r < end; r += blockDim.x) {
    row_token[r] = -1;
    row_scale[r] = 0.f;
  }
}

// Returns offsets [S+1], counts [S], row_of [n], row_token [cap], row_scale [cap].
std::vector<torch::Tensor> moe_plan(torch::Tensor idx, c10::optional<torch::Tensor> lut,
                                    c10::optional<torch::Tensor> weights, int64_t num_slots, int64_t capacity,
                                    int64_t align) {
  TORCH_CHECK(idx.is_cuda() && idx.scalar_type() == torch::kInt32 && idx.is_contiguous(), "idx int32");
  TORCH_CHECK(num_slots > 0 && num_slots <= 1024, "1..1024 slots");
  PM_CHECK_CUDA_OPT(lut); PM_CHECK_CUDA_OPT(weights);
  if (lut.has_value()) TORCH_CHECK(lut->scalar_type() == torch::kInt32 && lut->is_contiguous(), "lut int32");
  if (weights.has_value())
    TORCH_CHECK(weights->scalar_type() == torch::kFloat32 && weights->numel() == idx.numel(), "weights fp32");
  const int n = (int)idx.numel();
  const int K = (int)idx.size(-1);
  c10::cuda::CUDAGuard guard(idx.device());
  auto opt = idx.options();
  auto offsets = torch::empty({num_slots + 1}, opt);
  auto counts = torch::empty({num_slots}, opt);
  auto row_of = torch::empty({n}, opt);
  auto row_token = torch::empty({capacity}, opt);
  auto row_scale = torch::empty({capacity}, opt.dtype(torch::kFloat32));
  const int nblocks = std::max(1, (n + kPlanChunk - 1) / kPlanChunk);
  auto block_counts = torch::empty({nblocks, num_slots}, opt);
  auto stream = at::cuda::getCurrentCUDAStream();
  const int* lp = lut.has_value() ? lut->data_ptr<int>() : nullptr;
  const float* wp = weights.has_value() ? weights->data_ptr<float>() : nullptr;
  const int S = (int)num_slots;
  plan_count_kernel<<<nblocks, 256, S * sizeof(int), stream>>>(idx.data_ptr<int>(), lp, n, S,
                                                               block_counts.data_ptr<int>());
  plan_scan_kernel<<<1, 1024, 0, stream>>>(block_counts.data_ptr<int>(), nblocks, S, (int)align,
                                           offsets.data_ptr<int>(), counts.data_ptr<int>());
  const size_t smem = (size_t)kPlanWarps * S * sizeof(int);
  auto sk = plan_scatter_kernel;
  C10_CUDA_CHECK(cudaFuncSetAttribute(sk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  sk<<<nblocks, 256, smem, stream>>>(idx.data_ptr<int>(), lp, wp, n, K, S, block_counts.data_ptr<int>(),
                                     offsets.data_ptr<int>(), row_of.data_ptr<int>(), row_token.data_ptr<int>(),
                                     row_scale.data_ptr<float>());
  plan_pad_kernel<<<S, 128, 0, stream>>>(offsets.data_ptr<int>(), counts.data_ptr<int>(), S, row_token.data_ptr<int>(),
                                         row_scale.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {offsets, counts, row_of, row_token, row_scale};
}

// ----------------------------------------------------------------------------
// Row movement
// ----------------------------------------------------------------------------
// out[r] = src[row_token[r]] for r < offsets[S] (zero rows where row_token < 0)
__global__ void __launch_bounds__(256) gather_rows_kernel(const __nv_bfloat16* __restrict__ src, int nsrc,
                                                          const int* __restrict__ row_token,
                                                          const int* __restrict__ end_ptr, int cap, int H,
                                                          __nv_bfloat16* __restrict__ out) {
  const int end = end_ptr ? min(*end_ptr, cap) : cap;
  const int vec = H / 8;
  for (int r = blockIdx.x * 8 + (threadIdx.x >> 5); r < end; r += gridDim.x * 8) {
    const int t = row_token[r];
    uint4* o = reinterpret_cast<uint4*>(out + (size_t)r * H);
    if (t < 0 || !PM_INDEX_OK(t < nsrc)) {
      for (int i = threadIdx.x & 31; i < vec; i += 32) o[i] = make_uint4(0, 0, 0, 0);
    } else {
      const uint4* s = reinterpret_cast<const uint4*>(src + (size_t)t * H);
      for (int i = threadIdx.x & 31; i < vec; i += 32) o[i] = s[i];
    }
  }
}

// out[t] = sum_k src[row_of[t*K + k]]  (rows < 0 skipped), fp32 accumulation
__global__ void __launch_bounds__(256) sum_rows_kernel(const __nv_bfloat16* __restrict__ src, int nsrc,
                                                       const int* __restrict__ row_of, int T, int K, int H,
                                                       __nv_bfloat16* __restrict__ out) {
  const int vec = H / 8;
  for (int t = blockIdx.x * 8 + (threadIdx.x >> 5); t < T; t += gridDim.x * 8) {
    for (int i = threadIdx.x & 31; i < vec; i += 32) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int k = 0; k < K; ++k) {
        const int r = row_of[(size_t)t * K + k];
        if (r < 0 || !PM_INDEX_OK(r < nsrc)) continue;
        const uint4 q = reinterpret_cast<const uint4*>(src + (size_t)r * H)[i];
        const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[2 * j] += bf16_lo(u[j]);
          acc[2 * j + 1] += bf16_hi(u[j]);
        }
      }
      reinterpret_cast<uint4*>(out + (size_t)t * H)[i] =
          make_uint4(pack_bf16(acc[0], acc[1]), pack_bf16(acc[2], acc[3]), pack_bf16(acc[4], acc[5]),
                     pack_bf16(acc[6], acc[7]));
    }
  }
}

// out[a] = vals[row_of[a]] (0 where row_of < 0): per-assignment values from per-row values
__global__ void gather_scalar_kernel(const float* __restrict__ vals, int nvals, const int* __restrict__ row_of, int n,
                                     float* __restrict__ out) {
  const int a = blockIdx.x * blockDim.x + threadIdx.x;
  if (a < n) {
    const int r = row_of[a];
    out[a] = (r >= 0 && PM_INDEX_OK(r < nvals)) ? vals[r] : 0.f;
  }
}

static int sms() {
  int dev, n;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

void gather_rows(torch::Tensor src, torch::Tensor row_token, c10::optional<torch::Tensor> end, torch::Tensor out) {
  TORCH_CHECK(src.is_contiguous() && out.is_contiguous() && src.scalar_type() == torch::kBFloat16, "bf16 contiguous");
  const int H = (int)src.size(-1);
  TORCH_CHECK(H % 8 == 0 && out.size(-1) == H, "hidden");
  PM_CHECK_CUDA(src); PM_CHECK_CUDA(row_token); PM_CHECK_CUDA(out); PM_CHECK_CUDA_OPT(end);
  const int cap = (int)out.size(0);
  TORCH_CHECK(row_token.numel() >= cap, "row_token too short");
  TORCH_CHECK(row_token.is_contiguous() && row_token.scalar_type() == torch::kInt32, "row_token must be contiguous int32");
  c10::cuda::CUDAGuard guard(src.device());
  const int* ep = end.has_value() ? end->data_ptr<int>() : nullptr;
  const int grid = std::max(1, std::min((cap + 7) / 8, sms() * 8));
  gather_rows_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)src.data_ptr(), (int)src.size(0), row_token.data_ptr<int>(), ep, cap, H,
      (__nv_bfloat16*)out.data_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void sum_rows(torch::Tensor src, torch::Tensor row_of, torch::Tensor out) {
  TORCH_CHECK(src.is_contiguous() && out.is_contiguous(), "contiguous");
  TORCH_CHECK(row_of.is_contiguous() && row_of.scalar_type() == torch::kInt32, "row_of must be contiguous int32");
  PM_CHECK_CUDA(src); PM_CHECK_CUDA(row_of); PM_CHECK_CUDA(out);
  const int H = (int)src.size(-1);
  const int T = (int)out.size(0);
  const int K = (int)(row_of.numel() / std::max(T, 1));
  c10::cuda::CUDAGuard guard(src.device());
  if (T == 0) return;
  const int grid = std::max(1, std::min((T + 7) / 8, sms() * 8));
  sum_rows_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)src.data_ptr(), (int)src.size(0), row_of.data_ptr<int>(), T, K, H,
      (__nv_bfloat16*)out.data_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

torch::Tensor gather_scalar(torch::Tensor vals, torch::Tensor row_of) {
  PM_CHECK_CUDA(vals); PM_CHECK_CUDA(row_of);
  const int n = (int)row_of.numel();
  c10::cuda::CUDAGuard guard(vals.device());
  auto out = torch::empty(row_of.sizes(), vals.options());
  if (n == 0) return out;
  gather_scalar_kernel<<<(n + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      vals.data_ptr<float>(), (int)vals.numel(), row_of.data_ptr<int>(), n, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

}  // namespace pm

PM_DEFINE_ERROR_QUERY(pm_error_route)
