// RMSNorm and the fused QK-norm + RoPE kernels (sm_100a).
//
// rmsnorm_fwd/bwd: one warp per row, 16-byte vector accesses, fp32 math;
//   backward accumulates d(weight) per CTA in registers/shared memory and
//   adds it to the fp32 output with one atomic per element per CTA.
// qkv_rope_fwd/bwd: CTAs stride over tokens and split the fused QKV projection into
//   q/k/v, applies RMSNorm to q and k (groups of `q_group`/`k_group`
//   elements: head_dim for Qwen3-MoE per-head norms, the full width for
//   OLMoE), then rotary embedding (rotate-half convention) from a fp32
//   inverse-frequency table.
//
// Reference parity: RMSNorm/RoPE ops of veomni/ops/liger/__init__.py:52-133,
// veomni/ops/kernels/rms_norm/triton_batch_invariant.py:27 and the
// Qwen3-MoE attention of
// veomni/models/transformers/qwen3_moe/generated/patched_modeling_qwen3_moe_gpu.py.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace pm {

template <typename WT>
__device__ __forceinline__ float ldw(const WT* w, int i) { return static_cast<float>(w[i]); }
template <>
__device__ __forceinline__ float ldw<__nv_bfloat16>(const __nv_bfloat16* w, int i) { return __bfloat162float(w[i]); }

// H is a multiple of 256; each lane owns H/256 vectors of 8 elements.
template <int VPL, typename WT>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const WT* __restrict__ w,
                                                          __nv_bfloat16* __restrict__ y, float* __restrict__ rstd,
                                                          int rows, int H, float eps) {
  const int warp = (blockIdx.x * 8) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)warp * H);
  float v[VPL][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    uint4 q = xr[i * 32 + lane];
    uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[i][2 * j] = bf16_lo(u[j]);
      v[i][2 * j + 1] = bf16_hi(u[j]);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / H + eps);
  if (lane == 0) rstd[warp] = r;
  uint4* yr = reinterpret_cast<uint4*>(y + (size_t)warp * H);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c0 = (i * 32 + lane) * 8;
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      o[j] = pack_bf16(v[i][2 * j] * r * ldw(w, c0 + 2 * j), v[i][2 * j + 1] * r * ldw(w, c0 + 2 * j + 1));
    yr[i * 32 + lane] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <int VPL, typename WT>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                          const __nv_bfloat16* __restrict__ x, const WT* __restrict__ w,
                                                          const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dx,
                                                          float* __restrict__ dw, int rows, int H) {
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  float dwacc[VPL][8];
#pragma unroll
  for (int i = 0; i < VPL; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) dwacc[i][j] = 0.f;
  for (int row = blockIdx.x * 8 + wid; row < rows; row += gridDim.x * 8) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * H);
    const uint4* gr = reinterpret_cast<const uint4*>(dy + (size_t)row * H);
    const float r = rstd[row];
    float xv[VPL][8], gw[VPL][8];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      uint4 qx = xr[i * 32 + lane], qg = gr[i * 32 + lane];
      uint32_t ux[4] = {qx.x, qx.y, qx.z, qx.w}, ug[4] = {qg.x, qg.y, qg.z, qg.w};
      const int c0 = (i * 32 + lane) * 8;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        xv[i][2 * j] = bf16_lo(ux[j]);
        xv[i][2 * j + 1] = bf16_hi(ux[j]);
        const float g0 = bf16_lo(ug[j]), g1 = bf16_hi(ug[j]);
        dwacc[i][2 * j] += g0 * xv[i][2 * j] * r;
        dwacc[i][2 * j + 1] += g1 * xv[i][2 * j + 1] * r;
        gw[i][2 * j] = g0 * ldw(w, c0 + 2 * j);
        gw[i][2 * j + 1] = g1 * ldw(w, c0 + 2 * j + 1);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) dot += gw[i][j] * xv[i][j];
    }
    dot = warp_sum(dot);
    const float c = dot * r * r * r / H;
    uint4* dr = reinterpret_cast<uint4*>(dx + (size_t)row * H);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        o[j] = pack_bf16(r * gw[i][2 * j] - c * xv[i][2 * j], r * gw[i][2 * j + 1] - c * xv[i][2 * j + 1]);
      dr[i * 32 + lane] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  // reduce d(weight) over the 8 warps of the CTA, then one atomic per element
  extern __shared__ float sdw[];  // [H]
  for (int i = threadIdx.x; i < H; i += blockDim.x) sdw[i] = 0.f;
  __syncthreads();
#pragma unroll
  for (int i = 0; i < VPL; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) atomicAdd(&sdw[(i * 32 + lane) * 8 + j], dwacc[i][j]);
  __syncthreads();
  for (int i = threadIdx.x; i < H; i += blockDim.x) atomicAdd(&dw[i], sdw[i]);
}

static int sm_count() {
  int dev, n;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

#define PM_VPL_DISPATCH(H, ...)                                       \
  switch ((H) / 256) {                                               \
    case 1: { constexpr int VPL = 1; __VA_ARGS__; break; }           \
    case 2: { constexpr int VPL = 2; __VA_ARGS__; break; }           \
    case 4: { constexpr int VPL = 4; __VA_ARGS__; break; }           \
    case 8: { constexpr int VPL = 8; __VA_ARGS__; break; }           \
    case 16: { constexpr int VPL = 16; __VA_ARGS__; break; }         \
    default: TORCH_CHECK(false, "rmsnorm: hidden size must be 256 * {1,2,4,8,16}"); \
  }

std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, torch::Tensor w, double eps) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.is_contiguous(), "x must be contiguous bf16");
  const int H = (int)x.size(-1);
  const int rows = (int)(x.numel() / H);
  TORCH_CHECK(w.numel() == H && w.is_contiguous(), "weight size");
  PM_CHECK_CUDA(w);
  c10::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty_like(x);
  auto rstd = torch::empty({rows}, x.options().dtype(torch::kFloat32));
  if (rows == 0) return {y, rstd};
  auto stream = at::cuda::getCurrentCUDAStream();
  const int grid = (rows + 7) / 8;
  if (w.scalar_type() == torch::kFloat32) {
    PM_VPL_DISPATCH(H, rmsnorm_fwd_kernel<VPL, float><<<grid, 256, 0, stream>>>(
        (const __nv_bfloat16*)x.data_ptr(), w.data_ptr<float>(), (__nv_bfloat16*)y.data_ptr(),
        rstd.data_ptr<float>(), rows, H, (float)eps));
  } else {
    TORCH_CHECK(w.scalar_type() == torch::kBFloat16, "weight must be fp32 or bf16");
    PM_VPL_DISPATCH(H, rmsnorm_fwd_kernel<VPL, __nv_bfloat16><<<grid, 256, 0, stream>>>(
        (const __nv_bfloat16*)x.data_ptr(), (const __nv_bfloat16*)w.data_ptr(), (__nv_bfloat16*)y.data_ptr(),
        rstd.data_ptr<float>(), rows, H, (float)eps));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {y, rstd};
}

// returns dx (bf16) and accumulates into dw (fp32, [H])
torch::Tensor rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd, torch::Tensor dw) {
  TORCH_CHECK(dy.is_contiguous() && x.is_contiguous() && dy.scalar_type() == torch::kBFloat16, "dy/x contiguous bf16");
  TORCH_CHECK(dw.scalar_type() == torch::kFloat32 && dw.is_contiguous(), "dw must be fp32");
  PM_CHECK_CUDA(dy); PM_CHECK_CUDA(x); PM_CHECK_CUDA(w); PM_CHECK_CUDA(rstd); PM_CHECK_CUDA(dw);
  const int H = (int)x.size(-1);
  const int rows = (int)(x.numel() / H);
  c10::cuda::CUDAGuard guard(x.device());
  auto dx = torch::empty_like(x);
  if (rows == 0) return dx;
  auto stream = at::cuda::getCurrentCUDAStream();
  const int grid = std::min((rows + 7) / 8, sm_count() * 4);
  const size_t smem = (size_t)H * sizeof(float);
  if (w.scalar_type() == torch::kFloat32) {
    PM_VPL_DISPATCH(H, rmsnorm_bwd_kernel<VPL, float><<<grid, 256, smem, stream>>>(
        (const __nv_bfloat16*)dy.data_ptr(), (const __nv_bfloat16*)x.data_ptr(), w.data_ptr<float>(),
        rstd.data_ptr<float>(), (__nv_bfloat16*)dx.data_ptr(), dw.data_ptr<float>(), rows, H));
  } else {
    PM_VPL_DISPATCH(H, rmsnorm_bwd_kernel<VPL, __nv_bfloat16><<<grid, 256, smem, stream>>>(
        (const __nv_bfloat16*)dy.data_ptr(), (const __nv_bfloat16*)x.data_ptr(),
        (const __nv_bfloat16*)w.data_ptr(), rstd.data_ptr<float>(), (__nv_bfloat16*)dx.data_ptr(),
        dw.data_ptr<float>(), rows, H));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dx;
}

// ----------------------------------------------------------------------------
// Fused QK-norm + RoPE
// ----------------------------------------------------------------------------
struct QkvArgs {
  int T, Hq, Hkv, D;
  int q_group, k_group;  // RMSNorm group sizes (0 = no norm)
  float eps;
  const __nv_bfloat16* qkv;  // [T, (Hq + 2 Hkv) D]
  const int* pos;            // [T]
  const float* inv_freq;     // [D/2]
  const float* qw;           // [q_group] or null
  const float* kw;           // [k_group] or null
  __nv_bfloat16* q;          // [T, Hq, D]
  __nv_bfloat16* k;          // [T, Hkv, D]
  __nv_bfloat16* v;          // [T, Hkv, D]
  float* rq;                 // [T, Hq D / q_group]
  float* rk;                 // [T, Hkv D / k_group]
  // backward
  const __nv_bfloat16* dq;
  const __nv_bfloat16* dk;
  const __nv_bfloat16* dv;
  __nv_bfloat16* dqkv;
  float* dqw;
  float* dkw;
};

// Layout used by both kernels: warp w handles heads w, w + 8, ... (q heads then k
// heads, contiguous in the fused projection); lane l owns elements l + 32 c
// (c < D / 32) of each of its heads, so the RoPE partner of element c is
// c + D / 64 in the same lane.  Per-head norms reduce with warp shuffles; the
// full-width norm adds one block reduction.  No shared-memory atomics.
constexpr int kQkvWarps = 8;
constexpr int kMaxHeadsPerWarp = 8;  // (Hq + Hkv) <= 64

template <int D>
__global__ void __launch_bounds__(256) qkv_rope_fwd_kernel(QkvArgs a) {
  constexpr int C = D / 32;
  constexpr int HC = C / 2;
  __shared__ float red[2][kQkvWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NH = a.Hq + a.Hkv;
  const int width = (a.Hq + 2 * a.Hkv) * D;
  const int nq = a.Hq * D, nk = a.Hkv * D;
  const bool full_q = a.q_group > D, full_k = a.k_group > D;
  for (int t = blockIdx.x; t < a.T; t += gridDim.x) {
    const __nv_bfloat16* row = a.qkv + (size_t)t * width;
    float x[kMaxHeadsPerWarp][C];
    float ssq = 0.f, ssk = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxHeadsPerWarp; ++i) {
      const int h = warp + i * kQkvWarps;
      float s = 0.f;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        x[i][c] = h < NH ? __bfloat162float(row[h * D + lane + 32 * c]) : 0.f;
        s += x[i][c] * x[i][c];
      }
      if (h < a.Hq) ssq += s; else if (h < NH) ssk += s;
    }
    float rq_full = 1.f, rk_full = 1.f;
    if (full_q || full_k) {
      const float wq = warp_sum(ssq), wk = warp_sum(ssk);
      __syncthreads();
      if (lane == 0) { red[0][warp] = wq; red[1][warp] = wk; }
      __syncthreads();
      float tq = 0.f, tk = 0.f;
#pragma unroll
      for (int w = 0; w < kQkvWarps; ++w) { tq += red[0][w]; tk += red[1][w]; }
      rq_full = rsqrtf(tq / (float)(a.q_group ? a.q_group : 1) + a.eps);
      rk_full = rsqrtf(tk / (float)(a.k_group ? a.k_group : 1) + a.eps);
      if (threadIdx.x == 0) {
        if (full_q) a.rq[t] = rq_full;
        if (full_k) a.rk[t] = rk_full;
      }
    }
    const float p = (float)a.pos[t];
#pragma unroll
    for (int i = 0; i < kMaxHeadsPerWarp; ++i) {
      const int h = warp + i * kQkvWarps;
      if (h >= NH) continue;
      const bool isq = h < a.Hq;
      const int hl = isq ? h : h - a.Hq;  // head index within q or k
      const int G = isq ? a.q_group : a.k_group;
      const float* wt = isq ? a.qw : a.kw;
      float r = 1.f;
      if (G == D) {
        float s = 0.f;
#pragma unroll
        for (int c = 0; c < C; ++c) s += x[i][c] * x[i][c];
        r = rsqrtf(warp_sum(s) / (float)D + a.eps);
        if (lane == 0) (isq ? a.rq : a.rk)[(size_t)t * (isq ? a.Hq : a.Hkv) + hl] = r;
      } else if (G) {
        r = isq ? rq_full : rk_full;
      }
      float y[C];
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const int e = lane + 32 * c;
        const float wv = G == D ? wt[e] : (G ? wt[hl * D + e] : 1.f);
        y[c] = G ? x[i][c] * r * wv : x[i][c];
      }
      __nv_bfloat16* dst = isq ? a.q + ((size_t)t * a.Hq + hl) * D : a.k + ((size_t)t * a.Hkv + hl) * D;
#pragma unroll
      for (int c = 0; c < HC; ++c) {
        const int e = lane + 32 * c;
        float sn, cs;
        sincosf(p * a.inv_freq[e], &sn, &cs);
        dst[e] = __float2bfloat16(y[c] * cs - y[c + HC] * sn);
        dst[e + D / 2] = __float2bfloat16(y[c + HC] * cs + y[c] * sn);
      }
    }
    for (int i = threadIdx.x * 8; i < nk; i += blockDim.x * 8)
      *reinterpret_cast<uint4*>(a.v + (size_t)t * nk + i) = *reinterpret_cast<const uint4*>(row + nq + nk + i);
  }
}

template <int D>
__global__ void __launch_bounds__(256) qkv_rope_bwd_kernel(QkvArgs a) {
  constexpr int C = D / 32;
  constexpr int HC = C / 2;
  __shared__ float red[2][kQkvWarps];
  __shared__ float sdw[2][kQkvWarps][D];  // per-head norm weights: per-warp partials
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NH = a.Hq + a.Hkv;
  const int width = (a.Hq + 2 * a.Hkv) * D;
  const int nq = a.Hq * D, nk = a.Hkv * D;
  const bool full_q = a.q_group > D, full_k = a.k_group > D;
  float dwacc[kMaxHeadsPerWarp][C];
#pragma unroll
  for (int i = 0; i < kMaxHeadsPerWarp; ++i)
#pragma unroll
    for (int c = 0; c < C; ++c) dwacc[i][c] = 0.f;
  for (int t = blockIdx.x; t < a.T; t += gridDim.x) {
    const __nv_bfloat16* row = a.qkv + (size_t)t * width;
    __nv_bfloat16* drow = a.dqkv + (size_t)t * width;
    const float p = (float)a.pos[t];
    float x[kMaxHeadsPerWarp][C], g[kMaxHeadsPerWarp][C];
    float dotq = 0.f, dotk = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxHeadsPerWarp; ++i) {
      const int h = warp + i * kQkvWarps;
      if (h >= NH) {
#pragma unroll
        for (int c = 0; c < C; ++c) { x[i][c] = 0.f; g[i][c] = 0.f; }
        continue;
      }
      const bool isq = h < a.Hq;
      const int hl = isq ? h : h - a.Hq;
      const __nv_bfloat16* src = isq ? a.dq + ((size_t)t * a.Hq + hl) * D : a.dk + ((size_t)t * a.Hkv + hl) * D;
#pragma unroll
      for (int c = 0; c < HC; ++c) {
        const int e = lane + 32 * c;
        float sn, cs;
        sincosf(p * a.inv_freq[e], &sn, &cs);
        const float d0 = __bfloat162float(src[e]), d1 = __bfloat162float(src[e + D / 2]);
        g[i][c] = d0 * cs + d1 * sn;
        g[i][c + HC] = -d0 * sn + d1 * cs;
      }
      const int G = isq ? a.q_group : a.k_group;
      const float* wt = isq ? a.qw : a.kw;
      float dot = 0.f;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const int e = lane + 32 * c;
        x[i][c] = __bfloat162float(row[h * D + e]);
        const float wv = G == D ? wt[e] : (G ? wt[hl * D + e] : 1.f);
        dot += wv * g[i][c] * x[i][c];
      }
      if (G > D) { if (isq) dotq += dot; else dotk += dot; }
    }
    float tq = 0.f, tk = 0.f;
    if (full_q || full_k) {
      const float wq = warp_sum(dotq), wk = warp_sum(dotk);
      __syncthreads();
      if (lane == 0) { red[0][warp] = wq; red[1][warp] = wk; }
      __syncthreads();
#pragma unroll
      for (int w = 0; w < kQkvWarps; ++w) { tq += red[0][w]; tk += red[1][w]; }
    }
#pragma unroll
    for (int i = 0; i < kMaxHeadsPerWarp; ++i) {
      const int h = warp + i * kQkvWarps;
      if (h >= NH) continue;
      const bool isq = h < a.Hq;
      const int hl = isq ? h : h - a.Hq;
      const int G = isq ? a.q_group : a.k_group;
      const float* wt = isq ? a.qw : a.kw;
      __nv_bfloat16* dst = drow + h * D;
      if (!G) {
#pragma unroll
        for (int c = 0; c < C; ++c) dst[lane + 32 * c] = __float2bfloat16(g[i][c]);
        continue;
      }
      float r, dot;
      if (G == D) {
        r = (isq ? a.rq : a.rk)[(size_t)t * (isq ? a.Hq : a.Hkv) + hl];
        float d = 0.f;
#pragma unroll
        for (int c = 0; c < C; ++c) d += wt[lane + 32 * c] * g[i][c] * x[i][c];
        dot = warp_sum(d);
      } else {
        r = (isq ? a.rq : a.rk)[t];
        dot = isq ? tq : tk;
      }
      const float coef = r * r * r * dot / (float)G;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const int e = lane + 32 * c;
        const float wv = G == D ? wt[e] : wt[hl * D + e];
        dst[e] = __float2bfloat16(r * wv * g[i][c] - x[i][c] * coef);
        dwacc[i][c] += g[i][c] * x[i][c] * r;
      }
    }
    for (int i = threadIdx.x * 8; i < nk; i += blockDim.x * 8)
      *reinterpret_cast<uint4*>(drow + nq + nk + i) = *reinterpret_cast<const uint4*>(a.dv + (size_t)t * nk + i);
  }
  // weight gradients: full-width norms own one element per (head, lane, c) -> direct atomics;
  // per-head norms reduce over the warp's heads, then over the 8 warps in shared memory.
  float hq[C], hk[C];
#pragma unroll
  for (int c = 0; c < C; ++c) { hq[c] = 0.f; hk[c] = 0.f; }
#pragma unroll
  for (int i = 0; i < kMaxHeadsPerWarp; ++i) {
    const int h = warp + i * kQkvWarps;
    if (h >= NH) continue;
    const bool isq = h < a.Hq;
    const int hl = isq ? h : h - a.Hq;
    const int G = isq ? a.q_group : a.k_group;
    if (!G) continue;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const int e = lane + 32 * c;
      if (G == D) { if (isq) hq[c] += dwacc[i][c]; else hk[c] += dwacc[i][c]; }
      else atomicAdd(&(isq ? a.dqw : a.dkw)[hl * D + e], dwacc[i][c]);
    }
  }
  if (a.q_group == D || a.k_group == D) {
#pragma unroll
    for (int c = 0; c < C; ++c) { sdw[0][warp][lane + 32 * c] = hq[c]; sdw[1][warp][lane + 32 * c] = hk[c]; }
    __syncthreads();
    for (int e = threadIdx.x; e < 2 * D; e += blockDim.x) {
      const int which = e / D, j = e % D;
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kQkvWarps; ++w) s += sdw[which][w][j];
      if (which == 0 && a.q_group == D) atomicAdd(&a.dqw[j], s);
      if (which == 1 && a.k_group == D) atomicAdd(&a.dkw[j], s);
    }
  }
}

// Returns q [T,Hq,D], k [T,Hkv,D], v [T,Hkv,D], rstd_q, rstd_k.
std::vector<torch::Tensor> qkv_rope_fwd(torch::Tensor qkv, torch::Tensor pos, torch::Tensor inv_freq,
                                        c10::optional<torch::Tensor> qw, c10::optional<torch::Tensor> kw, int64_t Hq,
                                        int64_t Hkv, int64_t D, int64_t q_group, int64_t k_group, double eps) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == torch::kBFloat16 && qkv.is_contiguous(), "qkv contiguous bf16");
  TORCH_CHECK(qkv.size(-1) == (Hq + 2 * Hkv) * D, "qkv width");
  TORCH_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128");
  TORCH_CHECK(pos.scalar_type() == torch::kInt32 && inv_freq.scalar_type() == torch::kFloat32, "pos int32, inv_freq fp32");
  PM_CHECK_CUDA(pos); PM_CHECK_CUDA(inv_freq); PM_CHECK_CUDA_OPT(qw); PM_CHECK_CUDA_OPT(kw);
  TORCH_CHECK(!q_group || (qw.has_value() && qw->numel() == q_group), "q norm weight size");
  TORCH_CHECK(!k_group || (kw.has_value() && kw->numel() == k_group), "k norm weight size");
  const int T = (int)(qkv.numel() / qkv.size(-1));
  TORCH_CHECK(pos.numel() == T, "positions");
  c10::cuda::CUDAGuard guard(qkv.device());
  auto opt = qkv.options();
  auto q = torch::empty({T, Hq, D}, opt);
  auto k = torch::empty({T, Hkv, D}, opt);
  auto v = torch::empty({T, Hkv, D}, opt);
  const int qg = q_group ? (int)(Hq * D / q_group) : 0;
  const int kg = k_group ? (int)(Hkv * D / k_group) : 0;
  auto rq = torch::empty({T, std::max(qg, 1)}, opt.dtype(torch::kFloat32));
  auto rk = torch::empty({T, std::max(kg, 1)}, opt.dtype(torch::kFloat32));
  if (T == 0) return {q, k, v, rq, rk};
  QkvArgs a;
  memset(&a, 0, sizeof(a));
  a.T = T; a.Hq = (int)Hq; a.Hkv = (int)Hkv; a.D = (int)D; a.q_group = (int)q_group; a.k_group = (int)k_group;
  a.eps = (float)eps;
  a.qkv = (const __nv_bfloat16*)qkv.data_ptr(); a.pos = pos.data_ptr<int>(); a.inv_freq = inv_freq.data_ptr<float>();
  a.qw = q_group ? qw->data_ptr<float>() : nullptr;
  a.kw = k_group ? kw->data_ptr<float>() : nullptr;
  a.q = (__nv_bfloat16*)q.data_ptr(); a.k = (__nv_bfloat16*)k.data_ptr(); a.v = (__nv_bfloat16*)v.data_ptr();
  a.rq = rq.data_ptr<float>(); a.rk = rk.data_ptr<float>();
  TORCH_CHECK(Hq + Hkv <= kQkvWarps * kMaxHeadsPerWarp, "at most 64 q+k heads");
  TORCH_CHECK(!q_group || q_group == D || q_group == Hq * D, "q norm group: head_dim or full width");
  TORCH_CHECK(!k_group || k_group == D || k_group == Hkv * D, "k norm group: head_dim or full width");
  const int grid = std::min(T, sm_count() * 8);
  if (D == 128) qkv_rope_fwd_kernel<128><<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  else if (D == 64) qkv_rope_fwd_kernel<64><<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  else TORCH_CHECK(false, "head_dim must be 64 or 128");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {q, k, v, rq, rk};
}

// Returns dqkv; accumulates d(q_norm weight), d(k_norm weight) into dqw/dkw (fp32).
torch::Tensor qkv_rope_bwd(torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor qkv, torch::Tensor pos,
                           torch::Tensor inv_freq, c10::optional<torch::Tensor> qw, c10::optional<torch::Tensor> kw,
                           torch::Tensor rq, torch::Tensor rk, c10::optional<torch::Tensor> dqw,
                           c10::optional<torch::Tensor> dkw, int64_t Hq, int64_t Hkv, int64_t D, int64_t q_group,
                           int64_t k_group) {
  TORCH_CHECK(dq.is_contiguous() && dk.is_contiguous() && dv.is_contiguous(), "grads must be contiguous");
  PM_CHECK_CUDA(dq); PM_CHECK_CUDA(dk); PM_CHECK_CUDA(dv); PM_CHECK_CUDA(qkv); PM_CHECK_CUDA(pos);
  PM_CHECK_CUDA(inv_freq); PM_CHECK_CUDA(rq); PM_CHECK_CUDA(rk); PM_CHECK_CUDA_OPT(qw); PM_CHECK_CUDA_OPT(kw);
  PM_CHECK_CUDA_OPT(dqw); PM_CHECK_CUDA_OPT(dkw);
  const int T = (int)(qkv.numel() / qkv.size(-1));
  c10::cuda::CUDAGuard guard(qkv.device());
  auto dqkv = torch::empty_like(qkv);
  if (T == 0) return dqkv;
  const int qg = q_group ? (int)(Hq * D / q_group) : 0;
  const int kg = k_group ? (int)(Hkv * D / k_group) : 0;
  QkvArgs a;
  memset(&a, 0, sizeof(a));
  a.T = T; a.Hq = (int)Hq; a.Hkv = (int)Hkv; a.D = (int)D; a.q_group = (int)q_group; a.k_group = (int)k_group;
  a.qkv = (const __nv_bfloat16*)qkv.data_ptr(); a.pos = pos.data_ptr<int>(); a.inv_freq = inv_freq.data_ptr<float>();
  a.qw = q_group ? qw->data_ptr<float>() : nullptr;
  a.kw = k_group ? kw->data_ptr<float>() : nullptr;
  a.rq = rq.data_ptr<float>(); a.rk = rk.data_ptr<float>();
  a.dq = (const __nv_bfloat16*)dq.data_ptr(); a.dk = (const __nv_bfloat16*)dk.data_ptr();
  a.dv = (const __nv_bfloat16*)dv.data_ptr(); a.dqkv = (__nv_bfloat16*)dqkv.data_ptr();
  a.dqw = q_group ? dqw->data_ptr<float>() : nullptr;
  a.dkw = k_group ? dkw->data_ptr<float>() : nullptr;
  TORCH_CHECK(Hq + Hkv <= kQkvWarps * kMaxHeadsPerWarp, "at most 64 q+k heads");
  const int grid = std::min(T, sm_count() * 4);
  if (D == 128) qkv_rope_bwd_kernel<128><<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  else if (D == 64) qkv_rope_bwd_kernel<64><<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  else TORCH_CHECK(false, "head_dim must be 64 or 128");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dqkv;
}

}  // namespace pm

PM_DEFINE_ERROR_QUERY(pm_error_norm)
