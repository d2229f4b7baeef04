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
// PAIR variant (tcgen05 cta_group::2, clusters of 2 CTAs on 2 SMs): a tile is
// 256 x BN; CTA r of the pair loads rows [128r, 128r+128) of A and columns
// [BN/2 r, BN/2 (r+1)) of B into its own shared memory, the even CTA issues
// one 256 x BN MMA over both, and each CTA drains its own 128 accumulator
// rows.  Per SM this moves 2/3 of the operand bytes of a 128 x BN tile for
// the same tensor work.  Grouped-M segments must then be 256-row aligned.
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
constexpr int kThreads = 192;  // single-CTA tiles: TMA warp, MMA warp, 4 epilogue warps
constexpr int kMaxGroups = 256;  // bounded so that the deepest pipelines fit in 227 KB
constexpr int kEpiRing = 3;      // dSwiGLU: activation boxes in flight per epilogue warp

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
  const int* gather_idx;  // GATHER: source row of every A row (kGroupM) / B row (kGroupK); < 0 = padding
  int raster;       // 0: consecutive tiles walk M (B reused from L2); 1: walk N (A reused from L2)
};

template <int BN, int EPI = kStoreBF16, bool PAIR = false>
struct Cfg {
  static constexpr int kTM = PAIR ? 2 * BM : BM;     // tile rows (both CTAs)
  static constexpr int kBNc = PAIR ? BN / 2 : BN;    // B columns held by one CTA
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = kBNc * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  // Epilogue staging per CTA (4 warps): boxes of 32 rows handed to TMA stores.
  //   fp32 accumulate: 2 x 32x32 fp32 (4 KB) per warp; bf16 store: 2 x 32x32 bf16 (2 KB);
  //   SwiGLU: 2 x {h, gate, up} boxes; dSwiGLU: a ring of 4 {gate, up} boxes that TMA loads
  //   fill and the epilogue overwrites in place with d(gate), d(up) before storing them.
  static constexpr int kWarpStaging = EPI == kAccumF32 ? 2 * 4096
                                    : EPI == kStoreBF16 ? 2 * 2048
                                    : EPI == kSwiGLU ? 2 * 3 * 2048
                                    : EPI == kDSwiGLU ? kEpiRing * 2 * 2048 : 0;
  // pair tiles: two epilogue warps per TMEM lane quadrant, each draining half the columns
  static constexpr int kEpiWarps = PAIR ? 8 : 4;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr int kStagingBytes = kEpiWarps * kWarpStaging;
  static constexpr int kBudget = 224 * 1024;
  static constexpr int kStagesFit = (kBudget - kStagingBytes) / kStageBytes;
  static constexpr int kStages = kStagesFit > 6 ? 6 : kStagesFit;
  static_assert(kStages >= 3, "GEMM pipeline needs at least 3 stages");
  static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int kBarBytes = 512;
  static constexpr int kSmemBytes = kStages * kStageBytes + kStagingBytes + 1024 /*align*/ + kBarBytes;
};

struct TileInfo {
  int g;      // expert / group index (0 when ungrouped)
  int m0;     // first output row of the tile
  int n0;     // first output column of the tile
  int kbeg;   // first k index (rows of the token dim for kGroupK)
  int nkb;    // number of BK blocks
};

// Tile t -> coordinates.  ti.m0 is the first row owned by THIS CTA (the pair
// tile's first row + 128 * rank), n0 the tile's first output column.
template <int BN, int GROUP, bool SPLIT, int TM = BM>
__device__ __forceinline__ bool decode_tile(int t, const GemmArgs& a, const int* s_off, int total, TileInfo& ti,
                                            int crank = 0) {
  if (t >= total) return false;
  const int n_tiles = SPLIT ? (a.inter / (BN / 2)) : (a.N + BN - 1) / BN;
  if (GROUP == kGroupK) {
    const int m_tiles = (a.M + TM - 1) / TM;
    const int per = m_tiles * n_tiles;
    ti.g = t / per;
    const int r = t - ti.g * per;
    ti.n0 = (r / m_tiles) * BN;
    ti.m0 = (r % m_tiles) * TM + crank * BM;
    ti.kbeg = s_off[ti.g];
    ti.nkb = (s_off[ti.g + 1] - s_off[ti.g]) / BK;
  } else {
    int m_tiles;
    if (GROUP == kGroupM) m_tiles = s_off[a.num_groups] / TM;
    else m_tiles = (a.M + TM - 1) / TM;
    const int mt = a.raster ? t / n_tiles : t % m_tiles;
    const int nt = a.raster ? t % n_tiles : t / m_tiles;
    ti.m0 = mt * TM;
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
    ti.m0 += crank * BM;
  }
  return true;
}

template <int BN, int GROUP, bool SPLIT, int TM = BM>
__device__ __forceinline__ int total_tiles(const GemmArgs& a, const int* s_off) {
  const int n_tiles = SPLIT ? (a.inter / (BN / 2)) : (a.N + BN - 1) / BN;
  if (GROUP == kGroupK) return a.num_groups * ((a.M + TM - 1) / TM) * n_tiles;
  if (GROUP == kGroupM) return (s_off[a.num_groups] / TM) * n_tiles;
  return ((a.M + TM - 1) / TM) * n_tiles;
}

// Four gather indices (16-byte aligned); padding rows (< 0) read row 0, whose
// values are multiplied by zero routing weights / zero gradients downstream.
__device__ __forceinline__ int4 load_rows4(const int* p) {
  int4 r = *reinterpret_cast<const int4*>(p);
  r.x = max(r.x, 0); r.y = max(r.y, 0); r.z = max(r.z, 0); r.w = max(r.w, 0);
  return r;
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

template <int BN, bool A_MN, bool B_MN, int GROUP, int EPI, bool SPLIT, bool PAIR = false, bool GATHER = false>
__global__ void __launch_bounds__(Cfg<BN, EPI, PAIR>::kThreads, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmE,
                      GemmArgs args) {
  using C = Cfg<BN, EPI, PAIR>;
  constexpr int S = C::kStages;
  constexpr int TM = C::kTM;
  constexpr int BNc = C::kBNc;
  constexpr uint32_t kIdesc = make_idesc_bf16(TM, BN, A_MN, B_MN);
  // pair: CTA rank within the cluster, tile stride = number of pairs
  const int crank = PAIR ? (int)cluster_ctarank() : 0;
  const int first_tile = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tile_step = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

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
  uint64_t* ering = bars + 2 * S + 4;  // dSwiGLU: kEpiRing load barriers per epilogue warp
  static_assert((2 * 6 + 4 + 8 * kEpiRing) * 8 + 8 <= C::kBarBytes, "barrier area too small");
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 2 * S + 4 + C::kEpiWarps * kEpiRing);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  __shared__ int s_off[kMaxGroups + 1];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (GROUP != kGroupNone) {
    for (int i = threadIdx.x; i <= args.num_groups; i += C::kThreads) s_off[i] = args.group_offsets[i];
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
    // accumulator release: 4 epilogue warps (x 2 CTAs when paired, counted on the leader)
    for (int i = 0; i < 2; ++i) { mbar_init(&tfull[i], 1); mbar_init(&tempty[i], (PAIR ? 2 : 1) * C::kEpiWarps); }
    if (EPI == kDSwiGLU)
      for (int i = 0; i < C::kEpiWarps * kEpiRing; ++i) mbar_init(&ering[i], 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (EPI != kStoreF32) tma_prefetch_desc(&tmD);
    if (EPI == kSwiGLU || EPI == kDSwiGLU) tma_prefetch_desc(&tmE);
  }
  if (warp == 1) {
    if (PAIR) { tmem_alloc_pair(s_tmem, C::kTmemCols); tmem_relinquish_pair(); }
    else { tmem_alloc(s_tmem, C::kTmemCols); tmem_relinquish(); }
  }
  tc_fence_before();
  if (PAIR) cluster_sync();  // peer barriers initialised before any remote arrive / copy
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  int total = total_tiles<BN, GROUP, SPLIT, TM>(args, s_off);
  if (PAIR && GROUP == kGroupM) {
    // a 256-row pair tile must not straddle two experts: reject misaligned segment tables
    bool bad = false;
    for (int i = 0; i <= args.num_groups; ++i) bad |= (s_off[i] % TM) != 0;
    if (bad) {
      total = 0;
      if (threadIdx.x == 0) set_error(kErrArgs);
    }
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Lane 0 waits for free stages and issues the tiled loads.  With GATHER the
    // whole warp also issues row gathers: expert rows of A (kGroupM, lane l
    // fetches rows 4l..4l+3 of the CTA's 128) or token rows of B (kGroupK, lane
    // l fetches rows 4 (l % 16).. of the k-block into 64-column atom l / 16).
    static_assert(!GATHER || (GROUP == kGroupM && !A_MN) || (GROUP == kGroupK && B_MN && BNc % 128 == 0),
                  "gathered operand layout");
    if (lane == 0 || GATHER) {
      int s = 0; uint32_t ph = 0;
      int issued_mask = 0; uint32_t issued_par = 0;
      // paired: every copy completes on the leader's full barrier
      const uint32_t full0 = PAIR ? mapa_shared(smem_u32(&full[0]), 0) : 0u;
      TileInfo ti;
      for (int t = first_tile; decode_tile<BN, GROUP, SPLIT, TM>(t, args, s_off, total, ti, crank); t += tile_step) {
        int stop = *s_abort;
        if (GATHER) stop = __shfl_sync(0xffffffffu, stop, 0);  // the warp leaves together
        if (stop) break;
        // this CTA's B columns: the gate or up half (SPLIT), else its half of the tile
        const int nb = SPLIT ? (PAIR ? (crank ? args.inter + ti.n0 : ti.n0) : ti.n0) : ti.n0 + crank * BNc;
        int4 arow = make_int4(0, 0, 0, 0);
        if (GATHER && GROUP == kGroupM) arow = load_rows4(args.gather_idx + ti.m0 + 4 * lane);
        for (int kb = 0; kb < ti.nkb; ++kb) {
          bool free_ok = lane == 0 ? mbar_wait(&empty[s], ph ^ 1) : true;
          if (GATHER) free_ok = __shfl_sync(0xffffffffu, free_ok, 0);
          if (!free_ok) { if (lane == 0) *s_abort = 1; break; }
          const int k0 = ti.kbeg + kb * BK;
          uint8_t* a_dst = smA + s * C::kABytes;
          uint8_t* b_dst = smB + s * C::kBBytes;
          if (GATHER) {
            const uint32_t fb = PAIR ? full0 + (uint32_t)(s * sizeof(uint64_t)) : smem_u32(&full[s]);
            if (GROUP == kGroupM) {
              if (PAIR) tma_gather4_pair(a_dst + lane * 512, &tmA, fb, k0, arow);
              else tma_gather4(a_dst + lane * 512, &tmA, &full[s], k0, arow);
            } else {
              const int4 brow = load_rows4(args.gather_idx + k0 + 4 * (lane & 15));
#pragma unroll
              for (int at = lane >> 4; at < BNc / 64; at += 2) {
                uint8_t* dst = b_dst + at * 8192 + (lane & 15) * 512;
                if (PAIR) tma_gather4_pair(dst, &tmB, fb, nb + 64 * at, brow);
                else tma_gather4(dst, &tmB, &full[s], nb + 64 * at, brow);
              }
            }
          }
          if (lane != 0) {
            if (++s == S) { s = 0; ph ^= 1; }
            continue;
          }
          if (!PAIR || crank == 0) mbar_arrive_expect_tx(&full[s], (PAIR ? 2 : 1) * C::kStageBytes);
          if (PAIR) {
            const uint32_t fb = full0 + (uint32_t)(s * sizeof(uint64_t));
            if (GATHER && GROUP == kGroupM) {
              // A rows were gathered above
            } else if (!A_MN) {
              tma_load_2d_pair(a_dst, &tmA, fb, k0, ti.m0);
            } else {
              tma_load_2d_pair(a_dst, &tmA, fb, ti.m0, k0);
              tma_load_2d_pair(a_dst + 8192, &tmA, fb, ti.m0 + 64, k0);
            }
            if (GROUP == kGroupM) {
              if (!B_MN) {
                tma_load_3d_pair(b_dst, &tmB, fb, k0, nb, ti.g);
              } else {
#pragma unroll
                for (int j = 0; j < BNc / 64; ++j) tma_load_3d_pair(b_dst + j * 8192, &tmB, fb, nb + 64 * j, k0, ti.g);
              }
            } else if (!(GATHER && GROUP == kGroupK)) {
              if (!B_MN) {
                tma_load_2d_pair(b_dst, &tmB, fb, k0, nb);
              } else {
#pragma unroll
                for (int j = 0; j < BNc / 64; ++j) tma_load_2d_pair(b_dst + j * 8192, &tmB, fb, nb + 64 * j, k0);
              }
            }
          } else {
            if (GATHER && GROUP == kGroupM) {
              // A rows were gathered above
            } else if (!A_MN) {
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
            } else if (!(GATHER && GROUP == kGroupK)) {
              if (!B_MN) {
                tma_load_2d(b_dst, &tmB, &full[s], k0, ti.n0);
              } else {
#pragma unroll
                for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * 8192, &tmB, &full[s], ti.n0 + 64 * j, k0);
              }
            }
          }
          issued_mask |= 1 << s;
          issued_par = (issued_par & ~(1u << s)) | (ph << s);
          if (++s == S) { s = 0; ph ^= 1; }
        }
      }
      if (lane == 0 && *s_abort && (!PAIR || crank == 0)) {
        // Let copies already in flight land before the CTA exits (paired: the leader's
        // barriers count both CTAs' copies; the closing cluster barrier holds the peer).
        for (int i = 0; i < S; ++i)
          if (issued_mask & (1 << i)) mbar_wait(&full[i], (issued_par >> i) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0 && (!PAIR || crank == 0)) {
      int s = 0; uint32_t ph = 0;
      int acc = 0; uint32_t aph = 0;
      TileInfo ti;
      for (int t = first_tile; decode_tile<BN, GROUP, SPLIT, TM>(t, args, s_off, total, ti, crank); t += tile_step) {
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
            if (PAIR) umma_f16_pair(d_tmem, ad, bd, kIdesc, (kb | k) != 0);
            else umma_f16(d_tmem, ad, bd, kIdesc, (kb | k) != 0);
          }
          if (PAIR) umma_commit_pair(&empty[s], 3);
          else umma_commit(&empty[s]);
          if (++s == S) { s = 0; ph ^= 1; }
        }
        if (!ok) { *s_abort = 1; break; }
        if (PAIR) umma_commit_pair(&tfull[acc], 3);
        else umma_commit(&tfull[acc]);
        if (++acc == 2) { acc = 0; aph ^= 1; }
      }
    }
  } else {
    // ----------------------------------------------------------- epilogue
    // Each warp drains its TMEM lane quadrant (32 rows).  Results go through
    // swizzled shared-memory boxes of 32 rows and leave by TMA stores issued
    // from one lane (bulk groups; a box is rewritten only after its previous
    // store has read it).  bf16 boxes are 32 x 32 (64-byte rows, 64-byte
    // swizzle: 16-byte chunk j of row r sits at chunk j ^ ((r >> 1) & 3)).
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int r = q * 32 + lane;
    constexpr int kSplit = C::kEpiWarps / 4;  // warps sharing a quadrant split its columns
    const int half = (warp - 2) / 4;
    int acc = 0; uint32_t aph = 0;
    int epi_buf = 0;  // staging buffer toggle
    uint32_t ring_par = 0;      // dSwiGLU: parity bit per ring slot
    uint32_t ring_pending = 0;  // dSwiGLU: slots with a load in flight
    uint8_t* stg = staging + (warp - 2) * C::kWarpStaging;
    uint64_t* my_ring = ering + (warp - 2) * kEpiRing;
    const int sw64 = (lane >> 1) & 3;
    const uint32_t tempty0 = PAIR ? mapa_shared(smem_u32(&tempty[0]), 0) : 0u;
    TileInfo ti;
    for (int t = first_tile; decode_tile<BN, GROUP, SPLIT, TM>(t, args, s_off, total, ti, crank); t += tile_step) {
      if (*s_abort) break;
      const int y0 = ti.m0 + q * 32;  // first row of this warp's boxes
      constexpr int kChunks = BN / 32;
      // dSwiGLU: this warp's chunks are half, half + kSplit, ...; local index i counts them
      constexpr int kLocal = kChunks / kSplit;
      int issued = 0;
      if (EPI == kDSwiGLU) {
        // Start the saved-activation loads of this tile's first chunks while its mainloop runs.
        // Ring slots are free once every earlier store has read shared memory.
        constexpr int kFirst = kEpiRing - 1 < kLocal ? kEpiRing - 1 : kLocal;
        if (lane == 0) {
          bulk_wait_read_0();
          for (int i = 0; i < kFirst; ++i) {
            const int cc = half + i * kSplit;
            uint8_t* slot = stg + i * 4096;
            mbar_arrive_expect_tx(&my_ring[i], 4096);
            tma_load_2d(slot, &tmD, &my_ring[i], ti.n0 + cc * 32, y0);
            tma_load_2d(slot + 2048, &tmD, &my_ring[i], args.inter + ti.n0 + cc * 32, y0);
          }
        }
        issued = kFirst;
        ring_pending |= (1u << kFirst) - 1u;
      }
      if (!mbar_wait(&tfull[acc], aph)) { *s_abort = 1; break; }
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      const int row = ti.m0 + r;
      const bool empty_acc = ti.nkb == 0;

      if (EPI == kAccumF32) {
        // 32 x 32 fp32 boxes (128-byte rows, 128-byte swizzle): TMA reduce-add, or a TMA store
        // when beta == 0.
        const bool skip = empty_acc && args.beta == 1.0f;
#pragma unroll 1
        for (int c = half; c < kChunks && !skip; c += kSplit) {
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
      } else if (EPI == kStoreBF16) {
#pragma unroll 1
        for (int c = half; c < kChunks; c += kSplit) {
          const int col = ti.n0 + c * 32;
          if (col >= args.N) break;
          uint32_t rv[32];
          if (!empty_acc) { tmem_ld32(taddr + c * 32, rv); tmem_ld_wait(); }
          else {
#pragma unroll
            for (int i = 0; i < 32; ++i) rv[i] = 0u;
          }
          uint8_t* box = stg + (epi_buf & 1) * 2048;
          if (lane == 0) bulk_wait_read_1();
          __syncwarp();
          uint8_t* rowp = box + lane * 64;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            *reinterpret_cast<uint4*>(rowp + ((j ^ sw64) << 4)) = make_uint4(
                pack_bf16(__uint_as_float(rv[8 * j + 0]), __uint_as_float(rv[8 * j + 1])),
                pack_bf16(__uint_as_float(rv[8 * j + 2]), __uint_as_float(rv[8 * j + 3])),
                pack_bf16(__uint_as_float(rv[8 * j + 4]), __uint_as_float(rv[8 * j + 5])),
                pack_bf16(__uint_as_float(rv[8 * j + 6]), __uint_as_float(rv[8 * j + 7])));
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmD, box, col, y0);
            bulk_commit();
          }
          ++epi_buf;
        }
      } else if (EPI == kStoreF32) {
        // fp32 output (narrow router-logit GEMMs): direct row stores
        const bool row_ok = row < args.M;
        const size_t base_off = (size_t)row * args.ldd;
#pragma unroll 1
        for (int c = half; c < kChunks; c += kSplit) {
          uint32_t rv[32];
          if (!empty_acc) { tmem_ld32(taddr + c * 32, rv); tmem_ld_wait(); }
          else {
#pragma unroll
            for (int i = 0; i < 32; ++i) rv[i] = 0u;
          }
          const int col = ti.n0 + c * 32;
          const int valid = args.N - col;
          if (!row_ok || valid <= 0) continue;
          float* dst = reinterpret_cast<float*>(args.D) + base_off + col;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            if (4 * i >= valid) break;
            reinterpret_cast<float4*>(dst)[i] = make_float4(__uint_as_float(rv[4 * i]), __uint_as_float(rv[4 * i + 1]),
                                                            __uint_as_float(rv[4 * i + 2]),
                                                            __uint_as_float(rv[4 * i + 3]));
          }
        }
      } else if (EPI == kSwiGLU) {
        // tile columns [0, BN/2) are gate, [BN/2, BN) are up for output cols n0..n0+BN/2
        const float sc = args.row_scale ? args.row_scale[row] : 1.0f;
        const bool save = args.aux_out != nullptr;
#pragma unroll 1
        for (int c = half; c < BN / 64; c += kSplit) {
          uint32_t gv[32], uv[32];
          tmem_ld32(taddr + c * 32, gv);
          tmem_ld32(taddr + BN / 2 + c * 32, uv);
          tmem_ld_wait();
          const int col = ti.n0 + c * 32;
          uint8_t* set = stg + (epi_buf & 1) * 6144;  // h | gate | up boxes
          if (lane == 0) bulk_wait_read_1();
          __syncwarp();
          uint8_t* hrow = set + lane * 64;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float h[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float g = __uint_as_float(gv[8 * j + i]);
              h[i] = silu_f(g) * __uint_as_float(uv[8 * j + i]) * sc;
            }
            const int off = (j ^ sw64) << 4;
            *reinterpret_cast<uint4*>(hrow + off) =
                make_uint4(pack_bf16(h[0], h[1]), pack_bf16(h[2], h[3]), pack_bf16(h[4], h[5]), pack_bf16(h[6], h[7]));
            if (save) {
              *reinterpret_cast<uint4*>(hrow + 2048 + off) = make_uint4(
                  pack_bf16(__uint_as_float(gv[8 * j + 0]), __uint_as_float(gv[8 * j + 1])),
                  pack_bf16(__uint_as_float(gv[8 * j + 2]), __uint_as_float(gv[8 * j + 3])),
                  pack_bf16(__uint_as_float(gv[8 * j + 4]), __uint_as_float(gv[8 * j + 5])),
                  pack_bf16(__uint_as_float(gv[8 * j + 6]), __uint_as_float(gv[8 * j + 7])));
              *reinterpret_cast<uint4*>(hrow + 4096 + off) = make_uint4(
                  pack_bf16(__uint_as_float(uv[8 * j + 0]), __uint_as_float(uv[8 * j + 1])),
                  pack_bf16(__uint_as_float(uv[8 * j + 2]), __uint_as_float(uv[8 * j + 3])),
                  pack_bf16(__uint_as_float(uv[8 * j + 4]), __uint_as_float(uv[8 * j + 5])),
                  pack_bf16(__uint_as_float(uv[8 * j + 6]), __uint_as_float(uv[8 * j + 7])));
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmD, set, col, y0);
            if (save) {
              tma_store_2d(&tmE, set + 2048, col, y0);
              tma_store_2d(&tmE, set + 4096, args.inter + col, y0);
            }
            bulk_commit();
          }
          ++epi_buf;
        }
      } else if (EPI == kDSwiGLU) {
        // acc = dY * W2 for intermediate columns n0..n0+BN (unscaled by the routing weight).
        // Ring slot k holds the saved gate / up boxes of a chunk (TMA-loaded); after the chunk
        // is computed the slot is overwritten with d(gate) / d(up) and stored from there.
        const float sc = args.row_scale[row];
        float dw = 0.f;
        bool ok = true;
#pragma unroll 1
        for (int i = 0; i < kLocal; ++i) {
          const int c = half + i * kSplit;
          const int k = i % kEpiRing;
          uint8_t* slot = stg + k * 4096;
          if (!mbar_wait(&my_ring[k], (ring_par >> k) & 1)) { ok = false; break; }
          ring_par ^= 1u << k;
          ring_pending &= ~(1u << k);
          uint32_t rv[32];
          tmem_ld32(taddr + c * 32, rv);
          uint8_t* grow = slot + lane * 64;
          uint4 gq[4], uq[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            gq[j] = *reinterpret_cast<const uint4*>(grow + ((j ^ sw64) << 4));
            uq[j] = *reinterpret_cast<const uint4*>(grow + 2048 + ((j ^ sw64) << 4));
          }
          tmem_ld_wait();
          uint32_t dgp[16], dup[16];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t gw[4] = {gq[j].x, gq[j].y, gq[j].z, gq[j].w};
            const uint32_t uw[4] = {uq[j].x, uq[j].y, uq[j].z, uq[j].w};
#pragma unroll
            for (int h2 = 0; h2 < 4; ++h2) {
              float dgv[2], duv[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const float g = e ? bf16_hi(gw[h2]) : bf16_lo(gw[h2]);
                const float u = e ? bf16_hi(uw[h2]) : bf16_lo(uw[h2]);
                const float d = __uint_as_float(rv[8 * j + 2 * h2 + e]);
                const float sg = sigmoid_f(g);
                const float si = g * sg;
                dw += si * u * d;
                const float dh = d * sc;
                duv[e] = dh * si;
                dgv[e] = dh * u * sg * (1.0f + g * (1.0f - sg));
              }
              dgp[4 * j + h2] = pack_bf16(dgv[0], dgv[1]);
              dup[4 * j + h2] = pack_bf16(duv[0], duv[1]);
            }
          }
          __syncwarp();  // every lane has read the slot
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            *reinterpret_cast<uint4*>(grow + ((j ^ sw64) << 4)) =
                make_uint4(dgp[4 * j], dgp[4 * j + 1], dgp[4 * j + 2], dgp[4 * j + 3]);
            *reinterpret_cast<uint4*>(grow + 2048 + ((j ^ sw64) << 4)) =
                make_uint4(dup[4 * j], dup[4 * j + 1], dup[4 * j + 2], dup[4 * j + 3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int col = ti.n0 + c * 32;
            tma_store_2d(&tmE, slot, col, y0);
            tma_store_2d(&tmE, slot + 2048, args.inter + col, y0);
            bulk_commit();
            // refill the slot of this warp's previous chunk (its store was committed one chunk ago)
            if (issued < kLocal) {
              bulk_wait_read_1();
              const int kk = issued % kEpiRing;
              const int cc = half + issued * kSplit;
              uint8_t* ns = stg + kk * 4096;
              mbar_arrive_expect_tx(&my_ring[kk], 4096);
              tma_load_2d(ns, &tmD, &my_ring[kk], ti.n0 + cc * 32, y0);
              tma_load_2d(ns + 2048, &tmD, &my_ring[kk], args.inter + ti.n0 + cc * 32, y0);
            }
          }
          if (issued < kLocal) {
            ring_pending |= 1u << (issued % kEpiRing);
            ++issued;
          }
        }
        if (!ok) {
          *s_abort = 1;
          break;
        }
        if (args.row_grad) atomicAdd(&args.row_grad[row], dw);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR) mbar_arrive_cluster(tempty0 + (uint32_t)(acc * sizeof(uint64_t)));
        else mbar_arrive(&tempty[acc]);
      }
      if (++acc == 2) { acc = 0; aph ^= 1; }
    }
    // activation loads still in flight after an abort land before the CTA exits
    if (EPI == kDSwiGLU) {
      for (int k = 0; k < kEpiRing; ++k)
        if (ring_pending & (1u << k)) mbar_wait(&my_ring[k], (ring_par >> k) & 1);
    }
    // TMA stores / reductions read shared memory and write global memory asynchronously: drain them
    if (EPI != kStoreF32 && lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  if (PAIR) cluster_sync();  // neither CTA frees TMEM or exits while its peer still works
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR) tmem_dealloc_pair(tmem_base, C::kTmemCols);
    else tmem_dealloc(tmem_base, C::kTmemCols);
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

// grid: CTAs for the single-CTA kernel; for PAIR, the number of CTA pairs (launched as 2-CTA clusters).
template <int BN, bool A_MN, bool B_MN, int GROUP, int EPI, bool SPLIT, bool PAIR = false, bool GATHER = false>
static void launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args, int grid,
                   const CUtensorMap* td = nullptr, const CUtensorMap* te = nullptr) {
  using C = Cfg<BN, EPI, PAIR>;
  auto kern = gemm_sm100_kernel<BN, A_MN, B_MN, GROUP, EPI, SPLIT, PAIR, GATHER>;
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes));
    if (PAIR) C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0));
    configured = true;
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  CUtensorMap dummy;
  memset(&dummy, 0, sizeof(dummy));
  TORCH_CHECK(EPI == kStoreF32 || td != nullptr, "this GEMM epilogue needs an output tensor map");
  TORCH_CHECK(EPI != kDSwiGLU || te != nullptr, "dSwiGLU needs the d(gate|up) tensor map");
  TORCH_CHECK(EPI != kSwiGLU || te != nullptr || args.aux_out == nullptr, "SwiGLU save needs the gate|up tensor map");
  if (!PAIR) {
    kern<<<grid, C::kThreads, C::kSmemBytes, stream>>>(ta, tb, td ? *td : dummy, te ? *te : dummy, args);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(2 * grid, 1, 1);
  cfg.blockDim = dim3(C::kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, td ? *td : dummy, te ? *te : dummy, args));
}

// CTA pairs that can be resident at once (one pair per 2 SMs).
static inline int num_pairs() { return num_sms() / 2; }

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
