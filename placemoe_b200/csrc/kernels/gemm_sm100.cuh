// Persistent tcgen05 GEMM for sm_100a: dense and expert-grouped variants.
//
//   D[M, N] = sum_k A(m, k) * B(n, k)      (bf16 inputs, fp32 accumulation in TMEM)
//
// A is stored [M, K] (K-major) or [K, M] (MN-major); B is stored [N, K] or
// [K, N].  With both K-major this is Y = X W^T (forward); B MN-major gives
// the data gradient dX = dY W; both MN-major gives the weight gradient
// dW = dY^T X.
//
// Grouping (mixture-of-experts):
//   kGroupM  rows of A are expert segments whose offsets (multiples of 128)
//            live on the device; B is a stack of per-expert matrices.  Used for
//            expert forward and data gradients.  No host synchronisation:
//            the tile count is read from group_offsets[G] inside the kernel.
//   kGroupK  the contraction runs over each expert's token segment; each
//            expert writes its own output matrix.  Used for expert weight
//            gradients.
//
// Epilogues: bf16 store, fp32 store / accumulate, SwiGLU (gate/up halves of
// one tile, scaled by the per-row routing weight), dSwiGLU (recomputes the
// activation from the saved pre-activation and emits d(gate|up) plus the
// routing-weight gradient).
//
// Roles per CTA (192 threads): warp 0 issues TMA loads, warp 1 owns TMEM and
// issues tcgen05.mma from one lane, warps 2..5 drain the double-buffered
// accumulator from TMEM.  One CTA per SM; tiles are striped over the grid.
//
// Reference parity: replaces the Triton grouped GEMMs of
// veomni/ops/kernels/moe/_kernels/kernel/group_gemm.py:79 (same_nk) and :265
// (same_mn) and the EPGroupGemm autograd of
// veomni/distributed/moe/moe_layer.py:147.
#pragma once
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "tma.h"

namespace pm {

enum Epi : int { kStoreBF16 = 0, kStoreF32 = 1, kAccumF32 = 2, kSwiGLU = 3, kDSwiGLU = 4 };
enum Group : int { kGroupNone = 0, kGroupM = 1, kGroupK = 2 };

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;
constexpr int kMaxGroups = 512;

struct GemmArgs {
  int M, N, K;
  int num_groups;
  const int* group_offsets;  // [G+1] device, multiples of 128 (grouped modes)
  void* D;
  long long ldd;
  long long d_group_stride;  // kGroupK: elements between expert outputs
  const float* row_scale;    // SwiGLU / dSwiGLU: routing weight per row
  const __nv_bfloat16* aux;  // dSwiGLU: saved pre-activation [rows, 2I]
  long long ld_aux;
  __nv_bfloat16* aux_out;  // SwiGLU: optional pre-activation save; dSwiGLU: d(gate|up)
  long long ld_aux_out;
  float* row_grad;  // dSwiGLU: d(routing weight), atomically accumulated
  int inter;        // I: column offset of the "up" half
  float beta;       // kAccumF32: D = acc + beta * D
};

template <int BN, int EPI = kStoreBF16>
struct Cfg {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  // fp32-accumulating epilogues stage 32x32 fp32 boxes for TMA reduce-add: 4 warps x 2 buffers x 4 KB
  static constexpr int kStagingBytes = EPI == kAccumF32 ? 4 * 2 * 4096 : 0;
  static constexpr int kStages = EPI == kAccumF32 ? 3 : ((BN == 256) ? 4 : 6);
  static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int kSmemBytes = kStages * kStageBytes + kStagingBytes + 1024 /*align*/ + 256 /*barriers*/;
};

struct TileInfo {
  int g;      // expert / group index (0 when ungrouped)
  int m0;     // first output row of the tile
  int n0;     // first output column of the tile
  int kbeg;   // first k index (rows of the token dim for kGroupK)
  int nkb;    // number of BK blocks
};

template <int BN, int GROUP, bool SPLIT>
__device__ __forceinline__ bool decode_tile(int t, const GemmArgs& a, const int* s_off, int total, TileInfo& ti) {
  if (t >= total) return false;
  const int n_tiles = SPLIT ? (a.inter / (BN / 2)) : (a.N + BN - 1) / BN;
  if (GROUP == kGroupK) {
    const int m_tiles = (a.M + BM - 1) / BM;
    const int per = m_tiles * n_tiles;
    ti.g = t / per;
    const int r = t - ti.g * per;
    ti.n0 = (r / m_tiles) * BN;
    ti.m0 = (r % m_tiles) * BM;
    ti.kbeg = s_off[ti.g];
    ti.nkb = (s_off[ti.g + 1] - s_off[ti.g]) / BK;
  } else {
    int m_tiles;
    if (GROUP == kGroupM) m_tiles = s_off[a.num_groups] / BM;
    else m_tiles = (a.M + BM - 1) / BM;
    const int mt = t % m_tiles;
    const int nt = t / m_tiles;
    ti.m0 = mt * BM;
    ti.n0 = nt * (SPLIT ? BN / 2 : BN);
    ti.kbeg = 0;
    ti.nkb = (a.K + BK - 1) / BK;
    ti.g = 0;
    if (GROUP == kGroupM) {
      // largest g with s_off[g] <= m0
      int lo = 0, hi = a.num_groups - 1;
      while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (s_off[mid] <= ti.m0) lo = mid; else hi = mid - 1;
      }
      ti.g = lo;
    }
  }
  return true;
}

template <int BN, int GROUP, bool SPLIT>
__device__ __forceinline__ int total_tiles(const GemmArgs& a, const int* s_off) {
  const int n_tiles = SPLIT ? (a.inter / (BN / 2)) : (a.N + BN - 1) / BN;
  if (GROUP == kGroupK) return a.num_groups * ((a.M + BM - 1) / BM) * n_tiles;
  if (GROUP == kGroupM) return (s_off[a.num_groups] / BM) * n_tiles;
  return ((a.M + BM - 1) / BM) * n_tiles;
}

// Store 32 fp32 values as bf16 at dst (16-byte aligned), masking columns >= limit.
__device__ __forceinline__ void store_row32_bf16(__nv_bfloat16* dst, const float* v, int valid) {
  uint32_t p[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) p[i] = pack_bf16(v[2 * i], v[2 * i + 1]);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
  if (valid >= 32) {
#pragma unroll
    for (int i = 0; i < 4; ++i) d4[i] = make_uint4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (8 * i < valid) d4[i] = make_uint4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
  }
}

__device__ __forceinline__ void load_row32_bf16(const __nv_bfloat16* src, float* v) {
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 q = s4[i];
    v[8 * i + 0] = bf16_lo(q.x); v[8 * i + 1] = bf16_hi(q.x);
    v[8 * i + 2] = bf16_lo(q.y); v[8 * i + 3] = bf16_hi(q.y);
    v[8 * i + 4] = bf16_lo(q.z); v[8 * i + 5] = bf16_hi(q.z);
    v[8 * i + 6] = bf16_lo(q.w); v[8 * i + 7] = bf16_hi(q.w);
  }
}

template <int BN, bool A_MN, bool B_MN, int GROUP, int EPI, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmD, GemmArgs args) {
  using C = Cfg<BN, EPI>;
  constexpr int S = C::kStages;
  constexpr uint32_t kIdesc = make_idesc_bf16(BM, BN, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* smA = smem;
  uint8_t* smB = smem + S * C::kABytes;
  uint8_t* staging = smem + S * C::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(staging + C::kStagingBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* tfull = bars + 2 * S;
  uint64_t* tempty = bars + 2 * S + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 2 * S + 4);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  __shared__ int s_off[kMaxGroups + 1];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (GROUP != kGroupNone) {
    for (int i = threadIdx.x; i <= args.num_groups; i += kThreads) s_off[i] = args.group_offsets[i];
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&tfull[i], 1); mbar_init(&tempty[i], 4); }
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&tmA); tma_prefetch_desc(&tmB); }
  if (warp == 1) { tmem_alloc(s_tmem, C::kTmemCols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  const int total = total_tiles<BN, GROUP, SPLIT>(args, s_off);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int s = 0; uint32_t ph = 0;
      int issued_mask = 0; uint32_t issued_par = 0;
      TileInfo ti;
      for (int t = blockIdx.x; decode_tile<BN, GROUP, SPLIT>(t, args, s_off, total, ti); t += gridDim.x) {
        if (*s_abort) break;
        for (int kb = 0; kb < ti.nkb; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1)) { *s_abort = 1; break; }
          mbar_arrive_expect_tx(&full[s], C::kStageBytes);
          const int k0 = ti.kbeg + kb * BK;
          uint8_t* a_dst = smA + s * C::kABytes;
          uint8_t* b_dst = smB + s * C::kBBytes;
          if (!A_MN) {
            tma_load_2d(a_dst, &tmA, &full[s], k0, ti.m0);
          } else {
            tma_load_2d(a_dst, &tmA, &full[s], ti.m0, k0);
            tma_load_2d(a_dst + 8192, &tmA, &full[s], ti.m0 + 64, k0);
          }
          if (GROUP == kGroupM) {
            if (!B_MN) {
              if (SPLIT) {
                tma_load_3d(b_dst, &tmB, &full[s], k0, ti.n0, ti.g);
                tma_load_3d(b_dst + (BN / 2) * 128, &tmB, &full[s], k0, args.inter + ti.n0, ti.g);
              } else {
                tma_load_3d(b_dst, &tmB, &full[s], k0, ti.n0, ti.g);
              }
            } else {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j) tma_load_3d(b_dst + j * 8192, &tmB, &full[s], ti.n0 + 64 * j, k0, ti.g);
            }
          } else {
            if (!B_MN) {
              tma_load_2d(b_dst, &tmB, &full[s], k0, ti.n0);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * 8192, &tmB, &full[s], ti.n0 + 64 * j, k0);
            }
          }
          issued_mask |= 1 << s;
          issued_par = (issued_par & ~(1u << s)) | (ph << s);
          if (++s == S) { s = 0; ph ^= 1; }
        }
      }
      if (*s_abort) {
        // Let copies already in flight land before the CTA exits.
        for (int i = 0; i < S; ++i)
          if (issued_mask & (1 << i)) mbar_wait(&full[i], (issued_par >> i) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      int s = 0; uint32_t ph = 0;
      int acc = 0; uint32_t aph = 0;
      TileInfo ti;
      for (int t = blockIdx.x; decode_tile<BN, GROUP, SPLIT>(t, args, s_off, total, ti); t += gridDim.x) {
        if (*s_abort) break;
        if (!mbar_wait(&tempty[acc], aph ^ 1)) { *s_abort = 1; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < ti.nkb; ++kb) {
          if (!mbar_wait(&full[s], ph)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smA + s * C::kABytes);
          const uint32_t b_addr = smem_u32(smB + s * C::kBBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? make_sdesc_sw128(a_addr + k * 2048, 8192, 1024)
                                     : make_sdesc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? make_sdesc_sw128(b_addr + k * 2048, 8192, 1024)
                                     : make_sdesc_sw128(b_addr + k * 32, 16, 1024);
            umma_f16(d_tmem, ad, bd, kIdesc, (kb | k) != 0);
          }
          umma_commit(&empty[s]);
          if (++s == S) { s = 0; ph ^= 1; }
        }
        if (!ok) { *s_abort = 1; break; }
        umma_commit(&tfull[acc]);
        if (++acc == 2) { acc = 0; aph ^= 1; }
      }
    }
  } else {
    // ----------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int r = q * 32 + lane;
    int acc = 0; uint32_t aph = 0;
    int epi_buf = 0;  // kAccumF32: staging buffer toggle
    TileInfo ti;
    for (int t = blockIdx.x; decode_tile<BN, GROUP, SPLIT>(t, args, s_off, total, ti); t += gridDim.x) {
      if (*s_abort) break;
      if (!mbar_wait(&tfull[acc], aph)) { *s_abort = 1; break; }
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      const int row = ti.m0 + r;
      const bool empty_acc = ti.nkb == 0;

      if (EPI == kAccumF32) {
        // 32 rows (this warp's TMEM quadrant) x 32 columns per box: stage in swizzled smem, then
        // one lane issues a TMA reduce-add (or a TMA store when beta == 0) into the fp32 output.
        uint8_t* stg = staging + (warp - 2) * 2 * 4096;
        const bool skip = empty_acc && args.beta == 1.0f;
#pragma unroll 1
        for (int c = 0; c < BN / 32 && !skip; ++c) {
          const int col = ti.n0 + c * 32;
          if (col >= args.N) break;
          uint32_t rv[32];
          if (!empty_acc) { tmem_ld32(taddr + c * 32, rv); tmem_ld_wait(); }
          else {
#pragma unroll
            for (int i = 0; i < 32; ++i) rv[i] = 0u;
          }
          uint8_t* box = stg + (epi_buf & 1) * 4096;
          if (lane == 0) bulk_wait_read_1();
          __syncwarp();
          uint8_t* rowp = box + lane * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<uint4*>(rowp + ((j ^ (lane & 7)) << 4)) =
                make_uint4(rv[4 * j], rv[4 * j + 1], rv[4 * j + 2], rv[4 * j + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int y0 = ti.m0 + q * 32;
            if (GROUP == kGroupK) {
              if (args.beta != 0.0f) tma_reduce_add_3d(&tmD, box, col, y0, ti.g);
              else tma_store_3d(&tmD, box, col, y0, ti.g);
            } else {
              if (args.beta != 0.0f) tma_reduce_add_2d(&tmD, box, col, y0);
              else tma_store_2d(&tmD, box, col, y0);
            }
            bulk_commit();
          }
          ++epi_buf;
        }
      } else if (EPI == kStoreBF16 || EPI == kStoreF32) {
        const bool row_ok = row < args.M;
        size_t base_off = (size_t)row * args.ldd;
        if (GROUP == kGroupK) base_off += (size_t)ti.g * args.d_group_stride;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t rv[32];
          if (!empty_acc) { tmem_ld32(taddr + c * 32, rv); tmem_ld_wait(); }
          else {
#pragma unroll
            for (int i = 0; i < 32; ++i) rv[i] = 0u;
          }
          const int col = ti.n0 + c * 32;
          const int valid = args.N - col;
          if (!row_ok || valid <= 0) continue;
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(rv[i]);
          if (EPI == kStoreBF16) {
            store_row32_bf16(reinterpret_cast<__nv_bfloat16*>(args.D) + base_off + col, v, valid);
          } else {
            float* dst = reinterpret_cast<float*>(args.D) + base_off + col;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              if (4 * i >= valid) break;
              reinterpret_cast<float4*>(dst)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            }
          }
        }
      } else if (EPI == kSwiGLU) {
        // tile columns [0, BN/2) are gate, [BN/2, BN) are up for output cols n0..n0+BN/2
        const float sc = args.row_scale ? args.row_scale[row] : 1.0f;
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(args.D) + (size_t)row * args.ldd;
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          uint32_t gv[32], uv[32];
          tmem_ld32(taddr + c * 32, gv);
          tmem_ld32(taddr + BN / 2 + c * 32, uv);
          tmem_ld_wait();
          float h[32], gf[32], uf[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            gf[i] = __uint_as_float(gv[i]);
            uf[i] = __uint_as_float(uv[i]);
            h[i] = silu_f(gf[i]) * uf[i] * sc;
          }
          const int col = ti.n0 + c * 32;
          store_row32_bf16(out + col, h, 32);
          if (args.aux_out) {
            __nv_bfloat16* sv = args.aux_out + (size_t)row * args.ld_aux_out;
            store_row32_bf16(sv + col, gf, 32);
            store_row32_bf16(sv + args.inter + col, uf, 32);
          }
        }
      } else if (EPI == kDSwiGLU) {
        // acc = dY * W2 for intermediate columns n0..n0+BN (unscaled by the routing weight)
        const float sc = args.row_scale[row];
        const __nv_bfloat16* gu = args.aux + (size_t)row * args.ld_aux;
        __nv_bfloat16* dgu = args.aux_out + (size_t)row * args.ld_aux_out;
        float dw = 0.f;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t rv[32];
          tmem_ld32(taddr + c * 32, rv);
          tmem_ld_wait();
          const int col = ti.n0 + c * 32;
          float g[32], u[32], dg[32], du[32];
          load_row32_bf16(gu + col, g);
          load_row32_bf16(gu + args.inter + col, u);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float d = __uint_as_float(rv[i]);
            const float sg = sigmoid_f(g[i]);
            const float si = g[i] * sg;
            dw += si * u[i] * d;
            const float dh = d * sc;
            du[i] = dh * si;
            dg[i] = dh * u[i] * sg * (1.0f + g[i] * (1.0f - sg));
          }
          store_row32_bf16(dgu + col, dg, 32);
          store_row32_bf16(dgu + args.inter + col, du, 32);
        }
        if (args.row_grad) atomicAdd(&args.row_grad[row], dw);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) { acc = 0; aph ^= 1; }
    }
    // TMA reductions read shared memory and write global memory asynchronously: drain them
    if (EPI == kAccumF32 && lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// --------------------------------------------------------------------------
// Host side
// --------------------------------------------------------------------------

static inline int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int BN, bool A_MN, bool B_MN, int GROUP, int EPI, bool SPLIT>
static void launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args, int grid,
                   const CUtensorMap* td = nullptr) {
  using C = Cfg<BN, EPI>;
  auto kern = gemm_sm100_kernel<BN, A_MN, B_MN, GROUP, EPI, SPLIT>;
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes));
    configured = true;
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  CUtensorMap dummy;
  memset(&dummy, 0, sizeof(dummy));
  TORCH_CHECK(EPI != kAccumF32 || td != nullptr, "fp32-accumulating GEMM needs an output tensor map");
  kern<<<grid, kThreads, C::kSmemBytes, stream>>>(ta, tb, td ? *td : dummy, args);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static inline void check_bf16_2d(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == torch::kBFloat16, name, " must be bf16");
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.stride(1) == 1, name, " must have unit inner stride");
  TORCH_CHECK((t.stride(0) * 2) % 16 == 0, name, " row stride must be a multiple of 16 bytes");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, name, " must be 16-byte aligned");
}

static inline GemmArgs blank_args() {
  GemmArgs a;
  memset(&a, 0, sizeof(a));
  return a;
}

}  // namespace pm
