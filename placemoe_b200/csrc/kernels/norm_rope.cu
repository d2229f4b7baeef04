// RMSNorm and the fused QK-norm + RoPE kernels (sm_100a).
//
// rmsnorm_fwd/bwd: persistent warp-per-row kernels that stream rows through a
//   shared-memory ring (cp.async.bulk + mbarrier), fp32 math; the backward
//   keeps d(weight) partials in registers and adds them to the fp32 output
//   with one atomic per element per CTA.  add_rmsnorm_fwd / rmsnorm_bwd_add fold
//   the decoder's residual add (forward) and the residual-gradient add (backward)
//   into the same pass.
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

// RMSNorm rows are streamed through shared memory: every warp owns rows
// gw, gw + NW, ... (NW = warps in the grid) and its lane 0 keeps up to S of
// them in flight with cp.async.bulk copies into a per-warp ring of stages,
// one mbarrier per stage.  Bytes in flight therefore live in shared memory,
// not registers, which is what a bandwidth-bound row op needs to cover HBM
// latency.  Lane l owns the 16-byte chunks l, l + 32, ... of a row (VPL of
// them), so a lane's d(weight) partials always belong to the same columns.
constexpr int kRowWarps = 8;
constexpr int kRowMaxStages = 4;
constexpr int kRowSmemBudget = 220 * 1024;
constexpr int kRowBarBytes = kRowWarps * kRowMaxStages * 8;

static int sm_count() {
  int dev, n;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

// Issue the bulk copies of `nt` bf16 rows (same row index, `nt` tensors) into stage s.
template <int NT>
__device__ __forceinline__ void row_issue(uint8_t* stage, uint64_t* bar, const __nv_bfloat16* const (&src)[NT],
                                          size_t row, int H) {
  const uint32_t rb = (uint32_t)H * 2;
  mbar_arrive_expect_tx(bar, rb * NT);
#pragma unroll
  for (int t = 0; t < NT; ++t) bulk_load(stage + t * rb, src[t] + row * H, rb, bar);
}

// ADD: the row is h = x + res (rounded to bf16, as a bf16 tensor add would), written to `h`, and
// normalised; the residual add before a norm then costs no separate pass over the rows.
template <int VPL, typename WT, bool ADD = false>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const WT* __restrict__ w,
                                                          __nv_bfloat16* __restrict__ y, float* __restrict__ rstd,
                                                          int rows, int H, float eps, int S,
                                                          const __nv_bfloat16* __restrict__ res,
                                                          __nv_bfloat16* __restrict__ h) {
  constexpr int NT = ADD ? 2 : 1;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NW = gridDim.x * kRowWarps, gw = blockIdx.x * kRowWarps + warp;
  const uint32_t rb = (uint32_t)H * 2;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * kRowMaxStages;
  float* ws = reinterpret_cast<float*>(smem + kRowBarBytes);
  uint8_t* ring = smem + kRowBarBytes + (size_t)H * 4 + (size_t)warp * S * NT * rb;
  const __nv_bfloat16* src[NT];
  src[0] = x;
  if constexpr (ADD) src[NT - 1] = res;
  for (int i = threadIdx.x; i < H; i += blockDim.x) ws[i] = ldw(w, i);
  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
    for (int s = 0; s < S && gw + s * NW < rows; ++s)
      row_issue<NT>(ring + s * NT * rb, &bars[s], src, gw + s * NW, H);
  }
  __syncthreads();
  for (int k = 0;; ++k) {
    const int row = gw + k * NW;
    if (row >= rows) break;
    const int s = k % S;
    // warp-uniform exit when the wait runs out of budget (error recorded)
    if (!__all_sync(0xffffffffu, mbar_wait(&bars[s], (k / S) & 1))) break;
    const uint4* xs = reinterpret_cast<const uint4*>(ring + s * NT * rb);
    uint4 q[VPL];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      q[i] = xs[i * 32 + lane];
      if constexpr (ADD) {
        const uint4 b = reinterpret_cast<const uint4*>(ring + s * NT * rb + rb)[i * 32 + lane];
        q[i] = make_uint4(pack_bf16(bf16_lo(q[i].x) + bf16_lo(b.x), bf16_hi(q[i].x) + bf16_hi(b.x)),
                          pack_bf16(bf16_lo(q[i].y) + bf16_lo(b.y), bf16_hi(q[i].y) + bf16_hi(b.y)),
                          pack_bf16(bf16_lo(q[i].z) + bf16_lo(b.z), bf16_hi(q[i].z) + bf16_hi(b.z)),
                          pack_bf16(bf16_lo(q[i].w) + bf16_lo(b.w), bf16_hi(q[i].w) + bf16_hi(b.w)));
        reinterpret_cast<uint4*>(h + (size_t)row * H)[i * 32 + lane] = q[i];
      }
      const uint32_t u[4] = {q[i].x, q[i].y, q[i].z, q[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = bf16_lo(u[j]), b = bf16_hi(u[j]);
        ss += a * a + b * b;
      }
    }
    __syncwarp();
    if (lane == 0 && row + S * NW < rows) row_issue<NT>(ring + s * NT * rb, &bars[s], src, row + S * NW, H);
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / H + eps);
    if (lane == 0) rstd[row] = r;
    uint4* yr = reinterpret_cast<uint4*>(y + (size_t)row * H);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = i * 32 + lane;
      const float4 w0 = reinterpret_cast<const float4*>(ws)[2 * c], w1 = reinterpret_cast<const float4*>(ws)[2 * c + 1];
      const uint32_t u[4] = {q[i].x, q[i].y, q[i].z, q[i].w};
      uint4 o;
      o.x = pack_bf16(bf16_lo(u[0]) * r * w0.x, bf16_hi(u[0]) * r * w0.y);
      o.y = pack_bf16(bf16_lo(u[1]) * r * w0.z, bf16_hi(u[1]) * r * w0.w);
      o.z = pack_bf16(bf16_lo(u[2]) * r * w1.x, bf16_hi(u[2]) * r * w1.y);
      o.w = pack_bf16(bf16_lo(u[3]) * r * w1.z, bf16_hi(u[3]) * r * w1.w);
      yr[c] = o;
    }
  }
}

// Backward: dx = r*(dy*w) - (sum(dy*w*x) * r^3 / H) * x and dw += dy*x*r per row.
// Stage s of a warp holds [x row | dy row]; d(weight) partials stay in
// registers over all rows of the warp, are summed over the CTA's warps in
// shared memory and added to the fp32 output with one atomic per column per CTA.
// ADD: dx also receives `dres`, the gradient that reaches the norm's input through the residual
// path (dx = norm backward + dres, one rounding), so no separate gradient add runs.
template <int VPL, typename WT, bool ADD = false>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                          const __nv_bfloat16* __restrict__ x, const WT* __restrict__ w,
                                                          const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dx,
                                                          float* __restrict__ dw, int rows, int H, int S,
                                                          const __nv_bfloat16* __restrict__ dres) {
  constexpr int NT = ADD ? 3 : 2;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NW = gridDim.x * kRowWarps, gw = blockIdx.x * kRowWarps + warp;
  const uint32_t rb = (uint32_t)H * 2;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * kRowMaxStages;
  float* ws = reinterpret_cast<float*>(smem + kRowBarBytes);
  float* sdw = ws + H;
  uint8_t* ring = smem + kRowBarBytes + (size_t)H * 8 + (size_t)warp * S * NT * rb;
  const __nv_bfloat16* src[NT];
  src[0] = x;
  src[1] = dy;
  if constexpr (ADD) src[NT - 1] = dres;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    ws[i] = ldw(w, i);
    sdw[i] = 0.f;
  }
  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
    for (int s = 0; s < S && gw + s * NW < rows; ++s)
      row_issue<NT>(ring + s * NT * rb, &bars[s], src, gw + s * NW, H);
  }
  __syncthreads();
  constexpr bool kKeep = VPL <= 8;
  constexpr int kAcc = kKeep ? VPL : 1;
  float dwacc[kAcc][8];
#pragma unroll
  for (int i = 0; i < kAcc; ++i)
#pragma unroll
    for (int e = 0; e < 8; ++e) dwacc[i][e] = 0.f;
  for (int k = 0;; ++k) {
    const int row = gw + k * NW;
    if (row >= rows) break;
    const int s = k % S;
    const float r = rstd[row];
    // warp-uniform exit when the wait runs out of budget (error recorded)
    if (!__all_sync(0xffffffffu, mbar_wait(&bars[s], (k / S) & 1))) break;
    const uint4* xs = reinterpret_cast<const uint4*>(ring + s * NT * rb);
    const uint4* gs = reinterpret_cast<const uint4*>(ring + s * NT * rb + rb);
    const uint4* rs = reinterpret_cast<const uint4*>(ring + s * NT * rb + 2 * rb);  // ADD only
    uint4 qx[VPL], qg[VPL];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = i * 32 + lane;
      qx[i] = xs[c];
      qg[i] = gs[c];
      const uint32_t ux[4] = {qx[i].x, qx[i].y, qx[i].z, qx[i].w}, ug[4] = {qg[i].x, qg[i].y, qg[i].z, qg[i].w};
#pragma unroll
      for (int e2 = 0; e2 < 4; ++e2) {
        const float x0 = bf16_lo(ux[e2]), x1 = bf16_hi(ux[e2]);
        const float g0 = bf16_lo(ug[e2]), g1 = bf16_hi(ug[e2]);
        const float2 wv = reinterpret_cast<const float2*>(ws)[4 * c + e2];
        dot += g0 * wv.x * x0 + g1 * wv.y * x1;
        if constexpr (kKeep) {
          dwacc[i][2 * e2] += g0 * x0 * r;
          dwacc[i][2 * e2 + 1] += g1 * x1 * r;
        } else {  // wide rows: shared-memory accumulation keeps the registers for the row
          atomicAdd(&sdw[8 * c + 2 * e2], g0 * x0 * r);
          atomicAdd(&sdw[8 * c + 2 * e2 + 1], g1 * x1 * r);
        }
      }
    }
    if constexpr (kKeep && !ADD) {
      __syncwarp();
      if (lane == 0 && row + S * NW < rows) row_issue<NT>(ring + s * NT * rb, &bars[s], src, row + S * NW, H);
    }
    dot = warp_sum(dot);
    if constexpr (ADD) __syncwarp();  // the stage is read again below: keep those loads after this point
    const float cf = dot * r * r * r / H;
    uint4* dr = reinterpret_cast<uint4*>(dx + (size_t)row * H);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = i * 32 + lane;
      if constexpr (!kKeep || ADD) {  // read the stage again instead of holding it in registers
        qx[i] = xs[c];
        qg[i] = gs[c];
      }
      const uint32_t ux[4] = {qx[i].x, qx[i].y, qx[i].z, qx[i].w}, ug[4] = {qg[i].x, qg[i].y, qg[i].z, qg[i].w};
      uint32_t o[4];
      uint32_t ur[4] = {0u, 0u, 0u, 0u};
      if constexpr (ADD) {
        const uint4 q = rs[c];
        ur[0] = q.x; ur[1] = q.y; ur[2] = q.z; ur[3] = q.w;
      }
#pragma unroll
      for (int e2 = 0; e2 < 4; ++e2) {
        const float2 wv = reinterpret_cast<const float2*>(ws)[4 * c + e2];
        float a = r * bf16_lo(ug[e2]) * wv.x - cf * bf16_lo(ux[e2]);
        float b = r * bf16_hi(ug[e2]) * wv.y - cf * bf16_hi(ux[e2]);
        if constexpr (ADD) {
          a += bf16_lo(ur[e2]);
          b += bf16_hi(ur[e2]);
        }
        o[e2] = pack_bf16(a, b);
      }
      dr[c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
    if constexpr (!kKeep || ADD) {
      __syncwarp();
      if (lane == 0 && row + S * NW < rows) row_issue<NT>(ring + s * NT * rb, &bars[s], src, row + S * NW, H);
    }
  }
  if constexpr (kKeep) {
#pragma unroll
    for (int i = 0; i < VPL; ++i)
#pragma unroll
      for (int e = 0; e < 8; ++e) atomicAdd(&sdw[8 * (i * 32 + lane) + e], dwacc[i][e]);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < H; i += blockDim.x) atomicAdd(&dw[i], sdw[i]);
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

// Stages per warp and the CTA's shared-memory bytes for `nt` streamed tensors.
static void row_stream_shape(int H, int nt, int fixed_floats, int* S, int* smem) {
  const int stage = nt * H * 2;
  const int fixed = kRowBarBytes + fixed_floats * H * 4;
  const int s = (kRowSmemBudget - fixed) / (kRowWarps * stage);
  TORCH_CHECK(s >= 1, "rmsnorm: hidden size too large for the shared-memory ring");
  *S = std::min(s, kRowMaxStages);
  *smem = fixed + kRowWarps * *S * stage;
}

static void check_row_ptr(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, " must be 16-byte aligned");
}

std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, torch::Tensor w, double eps) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.is_contiguous(), "x must be contiguous bf16");
  const int H = (int)x.size(-1);
  const int rows = (int)(x.numel() / H);
  TORCH_CHECK(w.numel() == H && w.is_contiguous(), "weight size");
  PM_CHECK_CUDA(w);
  check_row_ptr(x, "x");
  c10::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty_like(x);
  auto rstd = torch::empty({rows}, x.options().dtype(torch::kFloat32));
  if (rows == 0) return {y, rstd};
  auto stream = at::cuda::getCurrentCUDAStream();
  int S, smem;
  row_stream_shape(H, 1, 1, &S, &smem);
  const int grid = std::min(sm_count(), (rows + kRowWarps - 1) / kRowWarps);
#define PM_RMS_FWD(WT_, WPTR)                                                                                      \
  PM_VPL_DISPATCH(H, {                                                                                             \
    auto kern = rmsnorm_fwd_kernel<VPL, WT_>;                                                                      \
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));                 \
    kern<<<grid, 256, smem, stream>>>((const __nv_bfloat16*)x.data_ptr(), WPTR, (__nv_bfloat16*)y.data_ptr(),      \
                                      rstd.data_ptr<float>(), rows, H, (float)eps, S, nullptr, nullptr);           \
  })
  if (w.scalar_type() == torch::kFloat32) {
    PM_RMS_FWD(float, w.data_ptr<float>());
  } else {
    TORCH_CHECK(w.scalar_type() == torch::kBFloat16, "weight must be fp32 or bf16");
    PM_RMS_FWD(__nv_bfloat16, (const __nv_bfloat16*)w.data_ptr());
  }
#undef PM_RMS_FWD
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {y, rstd};
}

// returns dx (bf16) and accumulates into dw (fp32, [H])
torch::Tensor rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd, torch::Tensor dw) {
  TORCH_CHECK(dy.is_contiguous() && x.is_contiguous() && dy.scalar_type() == torch::kBFloat16 &&
                  x.scalar_type() == torch::kBFloat16, "dy/x contiguous bf16");
  TORCH_CHECK(dw.scalar_type() == torch::kFloat32 && dw.is_contiguous(), "dw must be fp32");
  PM_CHECK_CUDA(dy); PM_CHECK_CUDA(x); PM_CHECK_CUDA(w); PM_CHECK_CUDA(rstd); PM_CHECK_CUDA(dw);
  const int H = (int)x.size(-1);
  const int rows = (int)(x.numel() / H);
  TORCH_CHECK(dy.numel() == x.numel() && w.numel() == H && dw.numel() == H && rstd.numel() == rows,
              "rmsnorm_bwd: shapes");
  check_row_ptr(x, "x");
  check_row_ptr(dy, "dy");
  c10::cuda::CUDAGuard guard(x.device());
  auto dx = torch::empty_like(x);
  if (rows == 0) return dx;
  auto stream = at::cuda::getCurrentCUDAStream();
  int S, smem;
  row_stream_shape(H, 2, 2, &S, &smem);
  const int grid = std::min(sm_count(), (rows + kRowWarps - 1) / kRowWarps);
#define PM_RMS_BWD(WT_, WPTR)                                                                                  \
  PM_VPL_DISPATCH(H, {                                                                                         \
    auto kern = rmsnorm_bwd_kernel<VPL, WT_>;                                                                  \
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));             \
    kern<<<grid, 256, smem, stream>>>((const __nv_bfloat16*)dy.data_ptr(), (const __nv_bfloat16*)x.data_ptr(), \
                                      WPTR, rstd.data_ptr<float>(), (__nv_bfloat16*)dx.data_ptr(),             \
                                      dw.data_ptr<float>(), rows, H, S, nullptr);                              \
  })
  if (w.scalar_type() == torch::kFloat32) {
    PM_RMS_BWD(float, w.data_ptr<float>());
  } else {
    TORCH_CHECK(w.scalar_type() == torch::kBFloat16, "weight must be fp32 or bf16");
    PM_RMS_BWD(__nv_bfloat16, (const __nv_bfloat16*)w.data_ptr());
  }
#undef PM_RMS_BWD
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dx;
}

// h = x + res (bf16) and y = rmsnorm(h): returns {h, y, rstd}.
std::vector<torch::Tensor> add_rmsnorm_fwd(torch::Tensor x, torch::Tensor res, torch::Tensor w, double eps) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.is_contiguous(), "x must be contiguous bf16");
  TORCH_CHECK(res.sizes() == x.sizes() && res.scalar_type() == torch::kBFloat16 && res.is_contiguous(),
              "res must be contiguous bf16 of x's shape");
  PM_CHECK_CUDA(res);
  const int H = (int)x.size(-1);
  const int rows = (int)(x.numel() / H);
  TORCH_CHECK(w.numel() == H && w.is_contiguous(), "weight size");
  PM_CHECK_CUDA(w);
  check_row_ptr(x, "x");
  check_row_ptr(res, "res");
  c10::cuda::CUDAGuard guard(x.device());
  auto h = torch::empty_like(x);
  auto y = torch::empty_like(x);
  auto rstd = torch::empty({rows}, x.options().dtype(torch::kFloat32));
  if (rows == 0) return {h, y, rstd};
  auto stream = at::cuda::getCurrentCUDAStream();
  int S, smem;
  row_stream_shape(H, 2, 1, &S, &smem);
  const int grid = std::min(sm_count(), (rows + kRowWarps - 1) / kRowWarps);
#define PM_ADD_RMS_FWD(WT_, WPTR)                                                                                  \
  PM_VPL_DISPATCH(H, {                                                                                             \
    auto kern = rmsnorm_fwd_kernel<VPL, WT_, true>;                                                                \
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));                 \
    kern<<<grid, 256, smem, stream>>>((const __nv_bfloat16*)x.data_ptr(), WPTR, (__nv_bfloat16*)y.data_ptr(),      \
                                      rstd.data_ptr<float>(), rows, H, (float)eps, S,                              \
                                      (const __nv_bfloat16*)res.data_ptr(), (__nv_bfloat16*)h.data_ptr());         \
  })
  if (w.scalar_type() == torch::kFloat32) {
    PM_ADD_RMS_FWD(float, w.data_ptr<float>());
  } else {
    TORCH_CHECK(w.scalar_type() == torch::kBFloat16, "weight must be fp32 or bf16");
    PM_ADD_RMS_FWD(__nv_bfloat16, (const __nv_bfloat16*)w.data_ptr());
  }
#undef PM_ADD_RMS_FWD
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {h, y, rstd};
}

// rmsnorm backward whose dx also receives the residual-path gradient `dres`; accumulates into dw.
torch::Tensor rmsnorm_bwd_add(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd, torch::Tensor dw,
                              torch::Tensor dres) {
  TORCH_CHECK(dy.is_contiguous() && x.is_contiguous() && dy.scalar_type() == torch::kBFloat16 &&
                  x.scalar_type() == torch::kBFloat16, "dy/x contiguous bf16");
  TORCH_CHECK(dres.is_contiguous() && dres.scalar_type() == torch::kBFloat16 && dres.numel() == x.numel(),
              "dres contiguous bf16 of x's size");
  TORCH_CHECK(dw.scalar_type() == torch::kFloat32 && dw.is_contiguous(), "dw must be fp32");
  PM_CHECK_CUDA(dy); PM_CHECK_CUDA(x); PM_CHECK_CUDA(w); PM_CHECK_CUDA(rstd); PM_CHECK_CUDA(dw); PM_CHECK_CUDA(dres);
  const int H = (int)x.size(-1);
  const int rows = (int)(x.numel() / H);
  TORCH_CHECK(dy.numel() == x.numel() && w.numel() == H && dw.numel() == H && rstd.numel() == rows,
              "rmsnorm_bwd_add: shapes");
  check_row_ptr(x, "x");
  check_row_ptr(dy, "dy");
  check_row_ptr(dres, "dres");
  c10::cuda::CUDAGuard guard(x.device());
  if (kRowBarBytes + 2 * H * 4 + kRowWarps * 3 * H * 2 > kRowSmemBudget) {
    // rows too wide for a ring of three streamed rows per warp: the plain backward, then the add
    auto dx = rmsnorm_bwd(dy, x, w, rstd, dw);
    dx.add_(dres);
    return dx;
  }
  auto dx = torch::empty_like(x);
  if (rows == 0) return dx;
  auto stream = at::cuda::getCurrentCUDAStream();
  int S, smem;
  row_stream_shape(H, 3, 2, &S, &smem);
  const int grid = std::min(sm_count(), (rows + kRowWarps - 1) / kRowWarps);
#define PM_RMS_BWD_ADD(WT_, WPTR)                                                                              \
  PM_VPL_DISPATCH(H, {                                                                                         \
    auto kern = rmsnorm_bwd_kernel<VPL, WT_, true>;                                                            \
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));             \
    kern<<<grid, 256, smem, stream>>>((const __nv_bfloat16*)dy.data_ptr(), (const __nv_bfloat16*)x.data_ptr(), \
                                      WPTR, rstd.data_ptr<float>(), (__nv_bfloat16*)dx.data_ptr(),             \
                                      dw.data_ptr<float>(), rows, H, S, (const __nv_bfloat16*)dres.data_ptr()); \
  })
  if (w.scalar_type() == torch::kFloat32) {
    PM_RMS_BWD_ADD(float, w.data_ptr<float>());
  } else {
    TORCH_CHECK(w.scalar_type() == torch::kBFloat16, "weight must be fp32 or bf16");
    PM_RMS_BWD_ADD(__nv_bfloat16, (const __nv_bfloat16*)w.data_ptr());
  }
#undef PM_RMS_BWD_ADD
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

// One block of 256 threads per token (persistent grid).  Thread j owns 16-byte
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

// Token ring: CTA b handles tokens b, b + G, ... (G = grid size); thread 0
// keeps S of them in flight with cp.async.bulk copies into shared-memory
// stages (one mbarrier each) and refills a stage once every thread of the
// CTA has read it.  A wait that runs out of budget ends the CTA uniformly
// (__syncthreads_or) after recording the error.
constexpr int kQkvBarBytes = 128;

PM_DEVICE void qkv_issue_fwd(const QkvArgs& a, uint8_t* stage, uint64_t* bar, int t, int width) {
  const uint32_t rb = (uint32_t)width * 2;
  mbar_arrive_expect_tx(bar, rb);
  bulk_load(stage, a.qkv + (size_t)t * width, rb, bar);
}

// Backward stage: [q|k inputs (nq + nk)][dq (nq)][dk (nk)][dv (nk)], bf16.
PM_DEVICE void qkv_issue_bwd(const QkvArgs& a, uint8_t* stage, uint64_t* bar, int t, int nq, int nk) {
  const int width = nq + 2 * nk;
  mbar_arrive_expect_tx(bar, (uint32_t)(2 * nq + 3 * nk) * 2);
  bulk_load(stage, a.qkv + (size_t)t * width, (uint32_t)(nq + nk) * 2, bar);
  bulk_load(stage + (size_t)(nq + nk) * 2, a.dq + (size_t)t * nq, (uint32_t)nq * 2, bar);
  bulk_load(stage + (size_t)(2 * nq + nk) * 2, a.dk + (size_t)t * nk, (uint32_t)nk * 2, bar);
  bulk_load(stage + (size_t)(2 * nq + 2 * nk) * 2, a.dv + (size_t)t * nk, (uint32_t)nk * 2, bar);
}

template <int D, int MQ, int MK>
__global__ void __launch_bounds__(kQkvThreads) qkv_rope_fwd_kernel(QkvArgs a, int S) {
  extern __shared__ __align__(128) uint8_t qsm[];
  __shared__ float red[2][kQkvThreads / 32];
  const int j = threadIdx.x, lane = j & 31;
  const int nq = a.Hq * D, nk = a.Hkv * D;
  const int nqc = nq / 8, nkc = nk / 8;
  const int width = nq + 2 * nk;
  const int o = (8 * j) % D;  // offset of this thread's chunks inside their heads
  const bool first_half = o < D / 2;
  const int ai = o % (D / 2);  // rotation-angle index of the chunk's first element
  const bool full_q = a.q_group > D, full_k = a.k_group > D;
  uint64_t* bar = reinterpret_cast<uint64_t*>(qsm);
  uint8_t* ring = qsm + kQkvBarBytes;
  const size_t stage_bytes = (size_t)width * 2;
  const int G = gridDim.x;
  if (j == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bar[s], 1);
    fence_barrier_init();
    for (int s = 0; s < S && (int)blockIdx.x + s * G < a.T; ++s)
      qkv_issue_fwd(a, ring + s * stage_bytes, &bar[s], blockIdx.x + s * G, width);
  }
  __syncthreads();
  int p_next = blockIdx.x < a.T ? a.pos[blockIdx.x] : 0;
  for (int it = 0;; ++it) {
    const int t = blockIdx.x + it * G;
    if (t >= a.T) break;
    const int s = it % S;
    const __nv_bfloat16* row = reinterpret_cast<const __nv_bfloat16*>(ring + s * stage_bytes);
    int p = p_next;
    if (t + (int)gridDim.x < a.T) p_next = a.pos[t + gridDim.x];  // next token's position in flight
    if (p < 0 || p >= a.rope_len) {
      if (j == 0) set_error(kErrBounds);
      p = 0;
    }
    float cs[8], sn[8];
    load_rope(a.rope + (size_t)p * (D / 2) + ai, cs, sn);
    const bool ok = mbar_wait(&bar[s], (it / S) & 1);
    if (__syncthreads_or(!ok)) break;
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
    for (int c = j; c < nkc; c += kQkvThreads)
      *reinterpret_cast<uint4*>(a.v + (size_t)t * nk + 8 * c) = *reinterpret_cast<const uint4*>(row + nq + nk + 8 * c);
    // every read of stage s is done once all threads passed the next barrier
    float rq_full = 1.f, rk_full = 1.f;
    if (full_q || full_k) {
      const float2 tot = block_sum2(tq, tk, red);
      rq_full = rsqrtf(tot.x / (float)(a.q_group ? a.q_group : 1) + a.eps);
      rk_full = rsqrtf(tot.y / (float)(a.k_group ? a.k_group : 1) + a.eps);
      if (j == 0) {
        if (full_q) a.rq[t] = rq_full;
        if (full_k) a.rk[t] = rk_full;
      }
    } else {
      __syncthreads();
    }
    if (j == 0 && t + S * G < a.T) qkv_issue_fwd(a, ring + s * stage_bytes, &bar[s], t + S * G, width);
#pragma unroll
    for (int i = 0; i < MQ; ++i)
      qkv_fwd_chunk<D>(xq[i], sq[i], j + kQkvThreads * i, nqc, a.q_group, a.qw, rq_full, a.rq, a.Hq, t,
                       a.q + (size_t)t * nq, cs, sn, o, first_half, a.eps, lane);
#pragma unroll
    for (int i = 0; i < MK; ++i)
      qkv_fwd_chunk<D>(xk[i], sk[i], j + kQkvThreads * i, nkc, a.k_group, a.kw, rk_full, a.rk, a.Hkv, t,
                       a.k + (size_t)t * nk, cs, sn, o, first_half, a.eps, lane);
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
                             int G, const float* wt, float r, __nv_bfloat16* dst, float (&dwa)[8], int o) {
  constexpr int HL = D / 8;
  float dx[8];
  if (!G) {
#pragma unroll
    for (int e = 0; e < 8; ++e) dx[e] = g[e];
  } else {
    const float dot = G == D ? head_sum<HL>(dot_part) : dot_full;
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
__global__ void __launch_bounds__(kQkvThreads) qkv_rope_bwd_kernel(QkvArgs a, int S) {
  extern __shared__ __align__(128) uint8_t qsm[];
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
  uint64_t* bar = reinterpret_cast<uint64_t*>(qsm);
  uint8_t* ring = qsm + kQkvBarBytes;
  const size_t stage_bytes = (size_t)(2 * nq + 3 * nk) * 2;
  const int G = gridDim.x;
  if (j == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bar[s], 1);
    fence_barrier_init();
    for (int s = 0; s < S && (int)blockIdx.x + s * G < a.T; ++s)
      qkv_issue_bwd(a, ring + s * stage_bytes, &bar[s], blockIdx.x + s * G, nq, nk);
  }
  __syncthreads();
  int p_next = blockIdx.x < a.T ? a.pos[blockIdx.x] : 0;
  for (int it = 0;; ++it) {
    const int t = blockIdx.x + it * G;
    if (t >= a.T) break;
    const int s = it % S;
    const __nv_bfloat16* row = reinterpret_cast<const __nv_bfloat16*>(ring + s * stage_bytes);
    const __nv_bfloat16* sdq = row + nq + nk;
    const __nv_bfloat16* sdk = sdq + nq;
    const __nv_bfloat16* sdv = sdk + nk;
    __nv_bfloat16* drow = a.dqkv + (size_t)t * width;
    int p = p_next;
    if (t + (int)gridDim.x < a.T) p_next = a.pos[t + gridDim.x];  // next token's position in flight
    if (p < 0 || p >= a.rope_len) {
      if (j == 0) set_error(kErrBounds);
      p = 0;
    }
    float cs[8], sn[8];
    load_rope(a.rope + (size_t)p * (D / 2) + ai, cs, sn);
    // saved inverse norms, loaded with the operands (not after the block reduction)
    float rq_s[MQ], rk_s[MK];
#pragma unroll
    for (int i = 0; i < MQ; ++i) {
      const int c = j + kQkvThreads * i;
      rq_s[i] = !a.q_group ? 0.f : (a.q_group == D ? (c < nqc ? a.rq[(size_t)t * a.Hq + (8 * c) / D] : 0.f) : a.rq[t]);
    }
#pragma unroll
    for (int i = 0; i < MK; ++i) {
      const int c = j + kQkvThreads * i;
      rk_s[i] = !a.k_group ? 0.f : (a.k_group == D ? (c < nkc ? a.rk[(size_t)t * a.Hkv + (8 * c) / D] : 0.f) : a.rk[t]);
    }
    const bool ok = mbar_wait(&bar[s], (it / S) & 1);
    if (__syncthreads_or(!ok)) break;
    float xq[MQ][8], gq[MQ][8], xk[MK][8], gk[MK][8], dq_h[MQ], dk_h[MK];
    float pq = 0.f, pk = 0.f;
#pragma unroll
    for (int i = 0; i < MQ; ++i) {
      dq_h[i] = qkv_bwd_load<D>(sdq, row, j + kQkvThreads * i, nqc, a.q_group, a.qw, xq[i], gq[i], cs, sn, o,
                                first_half);
      pq += dq_h[i];
    }
#pragma unroll
    for (int i = 0; i < MK; ++i) {
      dk_h[i] = qkv_bwd_load<D>(sdk, row + nq, j + kQkvThreads * i, nkc, a.k_group, a.kw, xk[i], gk[i], cs, sn, o,
                                first_half);
      pk += dk_h[i];
    }
    for (int c = j; c < nkc; c += kQkvThreads)
      *reinterpret_cast<uint4*>(drow + nq + nk + 8 * c) = *reinterpret_cast<const uint4*>(sdv + 8 * c);
    // every read of stage s is done once all threads passed the next barrier
    float tq = 0.f, tk = 0.f;
    if (full_q || full_k) {
      const float2 tot = block_sum2(pq, pk, red);
      tq = tot.x;
      tk = tot.y;
    } else {
      __syncthreads();
    }
    if (j == 0 && t + S * G < a.T) qkv_issue_bwd(a, ring + s * stage_bytes, &bar[s], t + S * G, nq, nk);
#pragma unroll
    for (int i = 0; i < MQ; ++i)
      qkv_bwd_store<D>(xq[i], gq[i], dq_h[i], tq, j + kQkvThreads * i, nqc, a.q_group, a.qw, rq_s[i], drow,
                       dwq[i], o);
#pragma unroll
    for (int i = 0; i < MK; ++i)
      qkv_bwd_store<D>(xk[i], gk[i], dk_h[i], tk, j + kQkvThreads * i, nkc, a.k_group, a.kw, rk_s[i], drow + nq,
                       dwk[i], o);
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

// Stages per CTA, dynamic shared memory and resident CTAs per SM for a ring of `stage` bytes.
template <typename K>
static void qkv_launch(K kern, int T, int stage, const QkvArgs& a) {
  int S = 3;
  while (S > 1 && kQkvBarBytes + S * stage > 160 * 1024) --S;
  const int smem = kQkvBarBytes + S * stage;
  TORCH_CHECK(smem <= 200 * 1024, "qkv rope: token row too wide for the shared-memory ring");
  C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  int per_sm = 0;
  C10_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kQkvThreads, smem));
  const int grid = std::min(T, sm_count() * std::max(per_sm, 1));
  kern<<<grid, kQkvThreads, smem, at::cuda::getCurrentCUDAStream()>>>(a, S);
}

#define PM_QKV_DISPATCH(KERNEL, D_, MQ_, MK_, T_, STAGE, ARGS)                                  \
  do {                                                                                          \
    if (D_ == 128) {                                                                            \
      if (MQ_ == 1 && MK_ == 1) qkv_launch(KERNEL<128, 1, 1>, T_, STAGE, ARGS);                 \
      else if (MQ_ == 2 && MK_ == 1) qkv_launch(KERNEL<128, 2, 1>, T_, STAGE, ARGS);            \
      else if (MQ_ <= 4 && MK_ == 1) qkv_launch(KERNEL<128, 4, 1>, T_, STAGE, ARGS);            \
      else qkv_launch(KERNEL<128, 4, 2>, T_, STAGE, ARGS);                                      \
    } else {                                                                                    \
      if (MQ_ == 1 && MK_ == 1) qkv_launch(KERNEL<64, 1, 1>, T_, STAGE, ARGS);                  \
      else if (MQ_ == 2 && MK_ == 1) qkv_launch(KERNEL<64, 2, 1>, T_, STAGE, ARGS);             \
      else if (MQ_ <= 4 && MK_ == 1) qkv_launch(KERNEL<64, 4, 1>, T_, STAGE, ARGS);             \
      else qkv_launch(KERNEL<64, 4, 2>, T_, STAGE, ARGS);                                       \
    }                                                                                           \
  } while (0)

static void check_aligned16(const torch::Tensor& t, const char* name) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, name, " must be 16-byte aligned");
}

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
  check_aligned16(qkv, "qkv");
  PM_QKV_DISPATCH(qkv_rope_fwd_kernel, D, mq, mk, T, (int)((Hq + 2 * Hkv) * D * 2), a);
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
  TORCH_CHECK(dq.scalar_type() == torch::kBFloat16 && dk.scalar_type() == torch::kBFloat16 &&
                  dv.scalar_type() == torch::kBFloat16 && qkv.scalar_type() == torch::kBFloat16,
              "qkv_rope_bwd: bf16 tensors");
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
  check_aligned16(qkv, "qkv");
  check_aligned16(dq, "dq");
  check_aligned16(dk, "dk");
  check_aligned16(dv, "dv");
  TORCH_CHECK(dq.numel() == (int64_t)T * Hq * D && dk.numel() == (int64_t)T * Hkv * D && dv.numel() == dk.numel(),
              "qkv_rope_bwd: gradient shapes");
  PM_QKV_DISPATCH(qkv_rope_bwd_kernel, D, mq, mk, T, (int)((2 * Hq + 3 * Hkv) * D * 2), a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dqkv;
}

}  // namespace pm

PM_DEFINE_ERROR_QUERY(pm_error_norm)
