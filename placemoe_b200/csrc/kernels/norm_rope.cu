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
  const float2* rope;        // [rope_len, D/2]: (cos, sin) of pos * inv_freq
  int rope_len;
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

// One block of 256 threads per token (grid-stride).  Thread j owns 16-byte
// chunks j, j + 256, ... of the q region and of the k region (8 consecutive
// elements each), so every global access is a 16-byte vector.  A head spans
// D / 8 consecutive threads; the RoPE partner of a chunk (offset +-D/2 in its
// head) lives in lane ^ (D / 16).  Per-head norms reduce over the head's lanes
// with shuffles, full-width norms with one block reduction per token.  The
// rotation angles come from a (cos, sin) table indexed by position.
constexpr int kQkvThreads = 256;

PM_DEVICE void load8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 q = *reinterpret_cast<const uint4*>(p);
  v[0] = bf16_lo(q.x); v[1] = bf16_hi(q.x); v[2] = bf16_lo(q.y); v[3] = bf16_hi(q.y);
  v[4] = bf16_lo(q.z); v[5] = bf16_hi(q.z); v[6] = bf16_lo(q.w); v[7] = bf16_hi(q.w);
}

PM_DEVICE void store8(__nv_bfloat16* p, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]),
                                            pack_bf16(v[6], v[7]));
}

PM_DEVICE void load8f(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

PM_DEVICE void load_rope(const float2* tab, float (&c)[8], float (&s)[8]) {
  const float4* t4 = reinterpret_cast<const float4*>(tab);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 v = t4[i];
    c[2 * i] = v.x; s[2 * i] = v.y; c[2 * i + 1] = v.z; s[2 * i + 1] = v.w;
  }
}

template <int HL>
PM_DEVICE float head_sum(float v) {
#pragma unroll
  for (int o = 1; o < HL; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum of two values over the block (all threads call it; returns the totals).
PM_DEVICE float2 block_sum2(float a, float b, float (*red)[kQkvThreads / 32]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  a = warp_sum(a);
  b = warp_sum(b);
  __syncthreads();
  if (lane == 0) { red[0][warp] = a; red[1][warp] = b; }
  __syncthreads();
  float ta = 0.f, tb = 0.f;
#pragma unroll
  for (int w = 0; w < kQkvThreads / 32; ++w) { ta += red[0][w]; tb += red[1][w]; }
  return make_float2(ta, tb);
}

// Normalise, rotate and store one chunk (forward).
template <int D>
PM_DEVICE void qkv_fwd_chunk(const float (&x)[8], float ssq, int c, int nch, int G, const float* wt, float rfull,
                             float* rsave, int H, int t, __nv_bfloat16* dst, const float (&cs)[8],
                             const float (&sn)[8], int o, bool first_half, float eps, int lane) {
  constexpr int HL = D / 8;
  constexpr int PX = D / 16;
  float r = 1.f;
  if (G == D) {
    r = rsqrtf(head_sum<HL>(ssq) / (float)D + eps);
    if (c < nch && (lane % HL) == 0) rsave[(size_t)t * H + (8 * c) / D] = r;
  } else if (G) {
    r = rfull;
  }
  float w8[8];
  if (G == D) load8f(wt + o, w8);
  else if (G && c < nch) load8f(wt + 8 * c, w8);
  else {
#pragma unroll
    for (int e = 0; e < 8; ++e) w8[e] = 1.f;
  }
  float y[8], out[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) y[e] = G ? x[e] * r * w8[e] : x[e];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float py = __shfl_xor_sync(0xffffffffu, y[e], PX);
    out[e] = first_half ? y[e] * cs[e] - py * sn[e] : y[e] * cs[e] + py * sn[e];
  }
  if (c < nch) store8(dst + 8 * c, out);
}

template <int D, int MQ, int MK>
__global__ void __launch_bounds__(kQkvThreads) qkv_rope_fwd_kernel(QkvArgs a) {
  __shared__ float red[2][kQkvThreads / 32];
  const int j = threadIdx.x, lane = j & 31;
  const int nq = a.Hq * D, nk = a.Hkv * D;
  const int nqc = nq / 8, nkc = nk / 8;
  const int width = nq + 2 * nk;
  const int o = (8 * j) % D;  // offset of this thread's chunks inside their heads
  const bool first_half = o < D / 2;
  const int ai = o % (D / 2);  // rotation-angle index of the chunk's first element
  const bool full_q = a.q_group > D, full_k = a.k_group > D;
  for (int t = blockIdx.x; t < a.T; t += gridDim.x) {
    const __nv_bfloat16* row = a.qkv + (size_t)t * width;
    int p = a.pos[t];
    if (p < 0 || p >= a.rope_len) {
      if (j == 0) set_error(kErrBounds);
      p = 0;
    }
    float cs[8], sn[8];
    load_rope(a.rope + (size_t)p * (D / 2) + ai, cs, sn);
    float xq[MQ][8], xk[MK][8], sq[MQ], sk[MK];
    float tq = 0.f, tk = 0.f;
#pragma unroll
    for (int i = 0; i < MQ; ++i) {
      const int c = j + kQkvThreads * i;
      if (c < nqc) load8(row + 8 * c, xq[i]);
      else {
#pragma unroll
        for (int e = 0; e < 8; ++e) xq[i][e] = 0.f;
      }
      sq[i] = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) sq[i] += xq[i][e] * xq[i][e];
      tq += sq[i];
    }
#pragma unroll
    for (int i = 0; i < MK; ++i) {
      const int c = j + kQkvThreads * i;
      if (c < nkc) load8(row + nq + 8 * c, xk[i]);
      else {
#pragma unroll
        for (int e = 0; e < 8; ++e) xk[i][e] = 0.f;
      }
      sk[i] = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) sk[i] += xk[i][e] * xk[i][e];
      tk += sk[i];
    }
    float rq_full = 1.f, rk_full = 1.f;
    if (full_q || full_k) {
      const float2 tot = block_sum2(tq, tk, red);
      rq_full = rsqrtf(tot.x / (float)(a.q_group ? a.q_group : 1) + a.eps);
      rk_full = rsqrtf(tot.y / (float)(a.k_group ? a.k_group : 1) + a.eps);
      if (j == 0) {
        if (full_q) a.rq[t] = rq_full;
        if (full_k) a.rk[t] = rk_full;
      }
    }
#pragma unroll
    for (int i = 0; i < MQ; ++i)
      qkv_fwd_chunk<D>(xq[i], sq[i], j + kQkvThreads * i, nqc, a.q_group, a.qw, rq_full, a.rq, a.Hq, t,
                       a.q + (size_t)t * nq, cs, sn, o, first_half, a.eps, lane);
#pragma unroll
    for (int i = 0; i < MK; ++i)
      qkv_fwd_chunk<D>(xk[i], sk[i], j + kQkvThreads * i, nkc, a.k_group, a.kw, rk_full, a.rk, a.Hkv, t,
                       a.k + (size_t)t * nk, cs, sn, o, first_half, a.eps, lane);
    for (int c = j; c < nkc; c += kQkvThreads)
      *reinterpret_cast<uint4*>(a.v + (size_t)t * nk + 8 * c) = *reinterpret_cast<const uint4*>(row + nq + nk + 8 * c);
  }
}

// Backward, phase 1 of a chunk: load, undo the rotation (g = R^T d), return the norm dot partial.
template <int D>
PM_DEVICE float qkv_bwd_load(const __nv_bfloat16* dsrc, const __nv_bfloat16* xsrc, int c, int nch, int G,
                             const float* wt, float (&x)[8], float (&g)[8], const float (&cs)[8],
                             const float (&sn)[8], int o, bool first_half) {
  constexpr int PX = D / 16;
  float d[8];
  if (c < nch) {
    load8(dsrc + 8 * c, d);
    load8(xsrc + 8 * c, x);
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) { d[e] = 0.f; x[e] = 0.f; }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float pd = __shfl_xor_sync(0xffffffffu, d[e], PX);
    g[e] = first_half ? d[e] * cs[e] + pd * sn[e] : d[e] * cs[e] - pd * sn[e];
  }
  float dot = 0.f;
  if (G && c < nch) {
    float w8[8];
    if (G == D) load8f(wt + o, w8);
    else load8f(wt + 8 * c, w8);
#pragma unroll
    for (int e = 0; e < 8; ++e) dot += w8[e] * g[e] * x[e];
  }
  return dot;
}

// Backward, phase 2 of a chunk: input gradient through the norm, weight-gradient partials.
template <int D>
PM_DEVICE void qkv_bwd_store(const float (&x)[8], const float (&g)[8], float dot_part, float dot_full, int c, int nch,
                             int G, const float* wt, const float* rsave, int H, int t, __nv_bfloat16* dst,
                             float (&dwa)[8], int o) {
  constexpr int HL = D / 8;
  float dx[8];
  if (!G) {
#pragma unroll
    for (int e = 0; e < 8; ++e) dx[e] = g[e];
  } else {
    float r, dot;
    if (G == D) {
      dot = head_sum<HL>(dot_part);
      r = c < nch ? rsave[(size_t)t * H + (8 * c) / D] : 0.f;
    } else {
      dot = dot_full;
      r = rsave[t];
    }
    float w8[8];
    if (G == D) load8f(wt + o, w8);
    else if (c < nch) load8f(wt + 8 * c, w8);
    else {
#pragma unroll
      for (int e = 0; e < 8; ++e) w8[e] = 0.f;
    }
    const float coef = r * r * r * dot / (float)G;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      dx[e] = r * w8[e] * g[e] - x[e] * coef;
      dwa[e] += g[e] * x[e] * r;
    }
  }
  if (c < nch) store8(dst + 8 * c, dx);
}

// Norm-weight gradient flush: full-width norms own distinct weights per chunk; per-head
// norms share weights o..o+7 across heads (summed over lanes, then warps in shared memory).
template <int D, int M>
PM_DEVICE void qkv_dw_flush(const float (&dwa)[M][8], int nch, int G, float* dw, float (*sdw_part)[D], int o) {
  constexpr int HL = D / 8;
  const int j = threadIdx.x, lane = j & 31, warp = j >> 5;
  if (!G || dw == nullptr) return;
  if (G > D) {
#pragma unroll
    for (int i = 0; i < M; ++i) {
      const int c = j + kQkvThreads * i;
      if (c < nch)
#pragma unroll
        for (int e = 0; e < 8; ++e) atomicAdd(&dw[8 * c + e], dwa[i][e]);
    }
    return;
  }
  float v[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    v[e] = 0.f;
#pragma unroll
    for (int i = 0; i < M; ++i) v[e] += dwa[i][e];
#pragma unroll
    for (int off = HL; off < 32; off <<= 1) v[e] += __shfl_xor_sync(0xffffffffu, v[e], off);
  }
  if (lane < HL) {
#pragma unroll
    for (int e = 0; e < 8; ++e) sdw_part[warp][o + e] = v[e];
  }
}

template <int D, int MQ, int MK>
__global__ void __launch_bounds__(kQkvThreads) qkv_rope_bwd_kernel(QkvArgs a) {
  constexpr int NW = kQkvThreads / 32;
  __shared__ float red[2][NW];
  __shared__ float sdw[2][NW][D];  // per-head norm weights: per-warp partials
  const int j = threadIdx.x;
  const int nq = a.Hq * D, nk = a.Hkv * D;
  const int nqc = nq / 8, nkc = nk / 8;
  const int width = nq + 2 * nk;
  const int o = (8 * j) % D;
  const bool first_half = o < D / 2;
  const int ai = o % (D / 2);
  const bool full_q = a.q_group > D, full_k = a.k_group > D;
  float dwq[MQ][8], dwk[MK][8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
#pragma unroll
    for (int i = 0; i < MQ; ++i) dwq[i][e] = 0.f;
#pragma unroll
    for (int i = 0; i < MK; ++i) dwk[i][e] = 0.f;
  }
  for (int t = blockIdx.x; t < a.T; t += gridDim.x) {
    const __nv_bfloat16* row = a.qkv + (size_t)t * width;
    __nv_bfloat16* drow = a.dqkv + (size_t)t * width;
    int p = a.pos[t];
    if (p < 0 || p >= a.rope_len) {
      if (j == 0) set_error(kErrBounds);
      p = 0;
    }
    float cs[8], sn[8];
    load_rope(a.rope + (size_t)p * (D / 2) + ai, cs, sn);
    float xq[MQ][8], gq[MQ][8], xk[MK][8], gk[MK][8], dq_h[MQ], dk_h[MK];
    float pq = 0.f, pk = 0.f;
#pragma unroll
    for (int i = 0; i < MQ; ++i) {
      dq_h[i] = qkv_bwd_load<D>(a.dq + (size_t)t * nq, row, j + kQkvThreads * i, nqc, a.q_group, a.qw, xq[i], gq[i],
                                cs, sn, o, first_half);
      pq += dq_h[i];
    }
#pragma unroll
    for (int i = 0; i < MK; ++i) {
      dk_h[i] = qkv_bwd_load<D>(a.dk + (size_t)t * nk, row + nq, j + kQkvThreads * i, nkc, a.k_group, a.kw, xk[i],
                                gk[i], cs, sn, o, first_half);
      pk += dk_h[i];
    }
    float tq = 0.f, tk = 0.f;
    if (full_q || full_k) {
      const float2 tot = block_sum2(pq, pk, red);
      tq = tot.x;
      tk = tot.y;
    }
#pragma unroll
    for (int i = 0; i < MQ; ++i)
      qkv_bwd_store<D>(xq[i], gq[i], dq_h[i], tq, j + kQkvThreads * i, nqc, a.q_group, a.qw, a.rq, a.Hq, t, drow,
                       dwq[i], o);
#pragma unroll
    for (int i = 0; i < MK; ++i)
      qkv_bwd_store<D>(xk[i], gk[i], dk_h[i], tk, j + kQkvThreads * i, nkc, a.k_group, a.kw, a.rk, a.Hkv, t,
                       drow + nq, dwk[i], o);
    for (int c = j; c < nkc; c += kQkvThreads)
      *reinterpret_cast<uint4*>(drow + nq + nk + 8 * c) = *reinterpret_cast<const uint4*>(a.dv + (size_t)t * nk + 8 * c);
  }
  qkv_dw_flush<D, MQ>(dwq, nqc, a.q_group, a.dqw, sdw[0], o);
  qkv_dw_flush<D, MK>(dwk, nkc, a.k_group, a.dkw, sdw[1], o);
  __syncthreads();
#pragma unroll
  for (int part = 0; part < 2; ++part) {
    const int G = part ? a.k_group : a.q_group;
    float* dw = part ? a.dkw : a.dqw;
    if (G != D || dw == nullptr) continue;
    for (int e = threadIdx.x; e < D; e += kQkvThreads) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) s += sdw[part][w][e];
      atomicAdd(&dw[e], s);
    }
  }
}

#define PM_QKV_DISPATCH(KERNEL, D_, MQ_, MK_, GRID, ARGS)                                              \
  do {                                                                                                 \
    auto st = at::cuda::getCurrentCUDAStream();                                                        \
    if (D_ == 128) {                                                                                   \
      if (MQ_ == 1 && MK_ == 1) KERNEL<128, 1, 1><<<GRID, kQkvThreads, 0, st>>>(ARGS);                 \
      else if (MQ_ == 2 && MK_ == 1) KERNEL<128, 2, 1><<<GRID, kQkvThreads, 0, st>>>(ARGS);            \
      else if (MQ_ <= 4 && MK_ == 1) KERNEL<128, 4, 1><<<GRID, kQkvThreads, 0, st>>>(ARGS);            \
      else KERNEL<128, 4, 2><<<GRID, kQkvThreads, 0, st>>>(ARGS);                                      \
    } else {                                                                                           \
      if (MQ_ == 1 && MK_ == 1) KERNEL<64, 1, 1><<<GRID, kQkvThreads, 0, st>>>(ARGS);                  \
      else if (MQ_ == 2 && MK_ == 1) KERNEL<64, 2, 1><<<GRID, kQkvThreads, 0, st>>>(ARGS);             \
      else if (MQ_ <= 4 && MK_ == 1) KERNEL<64, 4, 1><<<GRID, kQkvThreads, 0, st>>>(ARGS);             \
      else KERNEL<64, 4, 2><<<GRID, kQkvThreads, 0, st>>>(ARGS);                                       \
    }                                                                                                  \
  } while (0)

static void qkv_chunk_counts(int64_t Hq, int64_t Hkv, int64_t D, int& mq, int& mk) {
  const int64_t nqc = Hq * D / 8, nkc = Hkv * D / 8;
  TORCH_CHECK(nqc <= 4 * kQkvThreads, "q width must be at most ", 32 * kQkvThreads, " elements");
  TORCH_CHECK(nkc <= 2 * kQkvThreads, "k width must be at most ", 16 * kQkvThreads, " elements");
  mq = nqc <= kQkvThreads ? 1 : (nqc <= 2 * kQkvThreads ? 2 : 4);
  mk = nkc <= kQkvThreads ? 1 : 2;
}

static void check_rope_table(const torch::Tensor& rope, int64_t D) {
  TORCH_CHECK(rope.is_cuda() && rope.scalar_type() == torch::kFloat32 && rope.is_contiguous(), "rope table fp32");
  TORCH_CHECK(rope.dim() == 3 && rope.size(1) == D / 2 && rope.size(2) == 2, "rope table must be [L, D/2, 2]");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(rope.data_ptr()) & 15) == 0, "rope table must be 16-byte aligned");
}

// Returns q [T,Hq,D], k [T,Hkv,D], v [T,Hkv,D], rstd_q, rstd_k.
std::vector<torch::Tensor> qkv_rope_fwd(torch::Tensor qkv, torch::Tensor pos, torch::Tensor rope,
                                        c10::optional<torch::Tensor> qw, c10::optional<torch::Tensor> kw, int64_t Hq,
                                        int64_t Hkv, int64_t D, int64_t q_group, int64_t k_group, double eps) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == torch::kBFloat16 && qkv.is_contiguous(), "qkv contiguous bf16");
  TORCH_CHECK(qkv.size(-1) == (Hq + 2 * Hkv) * D, "qkv width");
  TORCH_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128");
  TORCH_CHECK(pos.scalar_type() == torch::kInt32, "pos must be int32");
  PM_CHECK_CUDA(pos); PM_CHECK_CUDA_OPT(qw); PM_CHECK_CUDA_OPT(kw);
  check_rope_table(rope, D);
  TORCH_CHECK(!q_group || (qw.has_value() && qw->numel() == q_group), "q norm weight size");
  TORCH_CHECK(!k_group || (kw.has_value() && kw->numel() == k_group), "k norm weight size");
  TORCH_CHECK(!q_group || q_group == D || q_group == Hq * D, "q norm group: head_dim or full width");
  TORCH_CHECK(!k_group || k_group == D || k_group == Hkv * D, "k norm group: head_dim or full width");
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
  a.qkv = (const __nv_bfloat16*)qkv.data_ptr(); a.pos = pos.data_ptr<int>();
  a.rope = reinterpret_cast<const float2*>(rope.data_ptr<float>()); a.rope_len = (int)rope.size(0);
  a.qw = q_group ? qw->data_ptr<float>() : nullptr;
  a.kw = k_group ? kw->data_ptr<float>() : nullptr;
  a.q = (__nv_bfloat16*)q.data_ptr(); a.k = (__nv_bfloat16*)k.data_ptr(); a.v = (__nv_bfloat16*)v.data_ptr();
  a.rq = rq.data_ptr<float>(); a.rk = rk.data_ptr<float>();
  int mq, mk;
  qkv_chunk_counts(Hq, Hkv, D, mq, mk);
  const int grid = std::min(T, sm_count() * 8);
  PM_QKV_DISPATCH(qkv_rope_fwd_kernel, D, mq, mk, grid, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {q, k, v, rq, rk};
}

// Returns dqkv; accumulates d(q_norm weight), d(k_norm weight) into dqw/dkw (fp32).
torch::Tensor qkv_rope_bwd(torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor qkv, torch::Tensor pos,
                           torch::Tensor rope, c10::optional<torch::Tensor> qw, c10::optional<torch::Tensor> kw,
                           torch::Tensor rq, torch::Tensor rk, c10::optional<torch::Tensor> dqw,
                           c10::optional<torch::Tensor> dkw, int64_t Hq, int64_t Hkv, int64_t D, int64_t q_group,
                           int64_t k_group) {
  TORCH_CHECK(dq.is_contiguous() && dk.is_contiguous() && dv.is_contiguous(), "grads must be contiguous");
  PM_CHECK_CUDA(dq); PM_CHECK_CUDA(dk); PM_CHECK_CUDA(dv); PM_CHECK_CUDA(qkv); PM_CHECK_CUDA(pos);
  PM_CHECK_CUDA(rq); PM_CHECK_CUDA(rk); PM_CHECK_CUDA_OPT(qw); PM_CHECK_CUDA_OPT(kw);
  PM_CHECK_CUDA_OPT(dqw); PM_CHECK_CUDA_OPT(dkw);
  check_rope_table(rope, D);
  TORCH_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128");
  const int T = (int)(qkv.numel() / qkv.size(-1));
  c10::cuda::CUDAGuard guard(qkv.device());
  auto dqkv = torch::empty_like(qkv);
  if (T == 0) return dqkv;
  QkvArgs a;
  memset(&a, 0, sizeof(a));
  a.T = T; a.Hq = (int)Hq; a.Hkv = (int)Hkv; a.D = (int)D; a.q_group = (int)q_group; a.k_group = (int)k_group;
  a.qkv = (const __nv_bfloat16*)qkv.data_ptr(); a.pos = pos.data_ptr<int>();
  a.rope = reinterpret_cast<const float2*>(rope.data_ptr<float>()); a.rope_len = (int)rope.size(0);
  a.qw = q_group ? qw->data_ptr<float>() : nullptr;
  a.kw = k_group ? kw->data_ptr<float>() : nullptr;
  a.rq = rq.data_ptr<float>(); a.rk = rk.data_ptr<float>();
  a.dq = (const __nv_bfloat16*)dq.data_ptr(); a.dk = (const __nv_bfloat16*)dk.data_ptr();
  a.dv = (const __nv_bfloat16*)dv.data_ptr(); a.dqkv = (__nv_bfloat16*)dqkv.data_ptr();
  a.dqw = q_group ? dqw->data_ptr<float>() : nullptr;
  a.dkw = k_group ? dkw->data_ptr<float>() : nullptr;
  int mq, mk;
  qkv_chunk_counts(Hq, Hkv, D, mq, mk);
  const int grid = std::min(T, sm_count() * 4);
  PM_QKV_DISPATCH(qkv_rope_bwd_kernel, D, mq, mk, grid, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dqkv;
}

}  // namespace pm

PM_DEFINE_ERROR_QUERY(pm_error_norm)
