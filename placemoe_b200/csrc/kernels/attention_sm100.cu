// Causal GQA flash attention on tcgen05 (sm_100a), forward and backward.
//
// Layout: q [T, Hq, D], k/v [T, Hkv, D], T = batch * seq_len, seq_len % 128 == 0,
// D in {64, 128}.  Tiles are 128 queries x 128 keys.  Optionally each row of seq_len
// tokens packs several documents: per-token document bounds mask keys of earlier
// documents (forward: the query's document start; backward: the key's document end).
//
// Forward, one CTA per (batch, q head, 128-query tile), 192 threads:
//   warp 0  TMA producer (Q once, K/V double-buffered)
//   warp 1  MMA issuer: S_j = Q K_j^T into one of two TMEM S buffers, then
//           O += P_{j-1} V_{j-1} once the softmax of tile j-1 is published,
//           so S_{j} overlaps softmax_{j-1}
//   warps 2-5  softmax: one query row per thread, online max/sum in fp32,
//           O rescaled in TMEM (skipped per warp when no row max moved), P
//           written bf16 into 128B-swizzled shared memory (the A operand).
//   TMEM: S0 | S1 | O   (512 columns allocated).
//
// Backward, one CTA per (batch, kv head, 128-key tile), looping over the q heads of
// the GQA group and the q tiles at or after the key tile: a warp-specialised
// pipeline (TMA warp, MMA warp, two compute warpgroups) in which P^T stays in
// TMEM as the A operand of dV += P^T dO, dQ tiles leave through TMA
// reduce-adds of swizzled fp32 staging boxes, and the MMAs of consecutive
// tiles overlap the elementwise work (details above the kernel).
//
// Reference parity: flash attention forward/backward used by
// veomni/ops/kernels/attention/__init__.py:151-353 (FA2/FA3/FA4 backends).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "tma.h"

namespace pm {

constexpr int kTile = 128;
constexpr int kAttnThreads = 192;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// K-major SW128 descriptor for a [rows x 128B-atom] tile; k-step of 16 elements
PM_DEVICE uint64_t kmaj_desc(uint32_t base, int kstep) {
  return make_sdesc_sw128(base + (kstep >> 2) * 16384 + (kstep & 3) * 32, 16, 1024);
}
// MN-major SW128 descriptor over a buffer made of 16 KB atoms (64 MN elements x 128 rows);
// k-step of 16 rows.
PM_DEVICE uint64_t mnmaj_desc(uint32_t base, int kstep) {
  return make_sdesc_sw128(base + kstep * 2048, 16384, 1024);
}

// write 8 packed bf16 (16 bytes) at chunk c of row r of a 128-row SW128 atom
PM_DEVICE void st_swz(uint8_t* atom, int r, int c, uint4 v) {
  *reinterpret_cast<uint4*>(atom + r * 128 + ((c ^ (r & 7)) << 4)) = v;
}

struct AttnArgs {
  int T, S, Hq, Hkv, B;
  float scale;  // 1/sqrt(D)
  __nv_bfloat16* o;
  float* lse;  // [Hq, T] natural-log LSE
  // backward
  const float* delta;  // [Hq, T]
  float* dq_acc;       // [T, Hq, D] fp32
  __nv_bfloat16* dk;   // [T, Hkv, D]
  __nv_bfloat16* dv;
  const float* lse_in;
  // packed documents (optional): per token, the first position of its document and the
  // position after its last token, both relative to the start of its row of seq_len tokens
  const int* doc_lo;
  const int* doc_hi;
};

// ---------------------------------------------------------------- forward
template <int D>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, AttnArgs a) {
  constexpr int ND = D / 64;           // 64-element atoms along D
  constexpr int kQBytes = ND * 16384;  // also K / V stage bytes
  constexpr uint32_t kIdescS = make_idesc_bf16(128, 128, false, false);
  constexpr uint32_t kIdescO = make_idesc_bf16(128, D, false, true);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sQ = sm;
  uint8_t* sK = sQ + kQBytes;           // 2 stages
  uint8_t* sV = sK + 2 * kQBytes;       // 2 stages
  uint8_t* sP = sV + 2 * kQBytes;       // 32 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 32768);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;     // [2]
  uint64_t* v_full = bars + 3;     // [2]
  uint64_t* kv_empty = bars + 5;   // [2]
  uint64_t* s_full = bars + 7;     // [2]
  uint64_t* s_free = bars + 9;     // [2]
  uint64_t* p_full = bars + 11;
  uint64_t* pv_done = bars + 12;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = a.S / kTile;
  const int L = blockIdx.x;
  const int qt = nq - 1 - L / (a.B * a.Hq);
  const int rem = L % (a.B * a.Hq);
  const int b = rem / a.Hq, h = rem % a.Hq;
  const int hk = h / (a.Hq / a.Hkv);
  const int tq0 = b * a.S + qt * kTile;
  const int nkv = qt + 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1); mbar_init(&v_full[i], 1); mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1); mbar_init(&s_free[i], 4);
    }
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) { tmem_alloc(s_tmem, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, kQBytes);
#pragma unroll
      for (int d = 0; d < ND; ++d) tma_load_3d(sQ + d * 16384, &tmQ, q_full, d * 64, h, tq0);
      for (int j = 0; j < nkv; ++j) {
        const int st = j & 1;
        if (!mbar_wait_abortable(&kv_empty[st], ((j >> 1) & 1) ^ 1, s_abort)) break;
        const int tk0 = b * a.S + j * kTile;
        mbar_arrive_expect_tx(&k_full[st], kQBytes);
#pragma unroll
        for (int d = 0; d < ND; ++d) tma_load_3d(sK + st * kQBytes + d * 16384, &tmK, &k_full[st], d * 64, hk, tk0);
        mbar_arrive_expect_tx(&v_full[st], kQBytes);
#pragma unroll
        for (int d = 0; d < ND; ++d) tma_load_3d(sV + st * kQBytes + d * 16384, &tmV, &v_full[st], d * 64, hk, tk0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t aq = smem_u32(sQ), ap = smem_u32(sP);
      const uint32_t t_o = tmem + 256;
      bool ok = mbar_wait_abortable(q_full, 0, s_abort);
      for (int j = 0; ok && j <= nkv; ++j) {
        if (j < nkv) {
          const int st = j & 1;
          if (!mbar_wait_abortable(&k_full[st], (j >> 1) & 1, s_abort)) break;
          if (!mbar_wait_abortable(&s_free[st], ((j >> 1) & 1) ^ 1, s_abort)) break;
          tc_fence_after();
          const uint32_t ak = smem_u32(sK + st * kQBytes);
#pragma unroll
          for (int k = 0; k < D / 16; ++k) umma_f16(tmem + st * 128, kmaj_desc(aq, k), kmaj_desc(ak, k), kIdescS, k > 0);
          umma_commit(&s_full[st]);
        }
        if (j >= 1) {
          const int pj = j - 1, st = pj & 1;
          if (!mbar_wait_abortable(p_full, pj & 1, s_abort)) break;
          if (!mbar_wait_abortable(&v_full[st], (pj >> 1) & 1, s_abort)) break;
          tc_fence_after();
          const uint32_t av = smem_u32(sV + st * kQBytes);
#pragma unroll
          for (int k = 0; k < 8; ++k) umma_f16(t_o, kmaj_desc(ap, k), mnmaj_desc(av, k), kIdescO, (pj > 0 || k > 0));
          umma_commit(&kv_empty[st]);
          umma_commit(pv_done);
        }
      }
    }
  } else {
    // softmax warps: one query row per thread
    const int qd = warp & 3;
    const int r = qd * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(qd * 32) << 16);
    const float c = a.scale * kLog2e;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int st = j & 1;
      if (!mbar_wait_abortable(&s_full[st], (j >> 1) & 1, s_abort)) { ok = false; break; }
      tc_fence_after();
      float x[128];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t v[32];
        tmem_ld32(trow + st * 128 + cc * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) x[cc * 32 + i] = __uint_as_float(v[i]) * c;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[st]);
      if (j == qt) {  // diagonal tile: key index > query index is masked
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i > r) x[i] = -INFINITY;
      }
      float mx = m;
#pragma unroll
      for (int i = 0; i < 128; ++i) mx = fmaxf(mx, x[i]);
      const float alpha = fast_exp2(m - mx);  // 0 on the first tile
      float rs = 0.f;
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        x[i] = fast_exp2(x[i] - mx);
        rs += x[i];
      }
      l = l * alpha + rs;
      m = mx;
      if (j > 0) {
        if (!mbar_wait_abortable(pv_done, (j - 1) & 1, s_abort)) { ok = false; break; }
        tc_fence_after();
        if (!__all_sync(0xffffffffu, alpha == 1.0f)) {
#pragma unroll
          for (int cc = 0; cc < D / 16; ++cc) {
            uint32_t v[16];
            tmem_ld16(trow + 256 + cc * 16, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
            tmem_st16(trow + 256 + cc * 16, v);
          }
          tmem_st_wait();
        }
      }
      // P (bf16) -> swizzled smem, 2 atoms of 64 keys
#pragma unroll
      for (int cch = 0; cch < 16; ++cch) {
        const int k0 = cch * 8;
        uint4 pk = make_uint4(pack_bf16(x[k0], x[k0 + 1]), pack_bf16(x[k0 + 2], x[k0 + 3]),
                              pack_bf16(x[k0 + 4], x[k0 + 5]), pack_bf16(x[k0 + 6], x[k0 + 7]));
        st_swz(sP + (cch >> 3) * 16384, r, cch & 7, pk);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && mbar_wait_abortable(pv_done, (nkv - 1) & 1, s_abort)) {
      tc_fence_after();
      const float inv = 1.f / l;
      __nv_bfloat16* orow = a.o + ((size_t)(tq0 + r) * a.Hq + h) * D;
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t v[32];
        tmem_ld32(trow + 256 + cc * 32, v);
        tmem_ld_wait();
        uint4* dst = reinterpret_cast<uint4*>(orow + cc * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          dst[i] = make_uint4(pack_bf16(__uint_as_float(v[8 * i]) * inv, __uint_as_float(v[8 * i + 1]) * inv),
                              pack_bf16(__uint_as_float(v[8 * i + 2]) * inv, __uint_as_float(v[8 * i + 3]) * inv),
                              pack_bf16(__uint_as_float(v[8 * i + 4]) * inv, __uint_as_float(v[8 * i + 5]) * inv),
                              pack_bf16(__uint_as_float(v[8 * i + 6]) * inv, __uint_as_float(v[8 * i + 7]) * inv));
      }
      a.lse[(size_t)h * a.T + tq0 + r] = (m + __log2f(l)) * kLn2;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// 2^x for x <= 0 on the FMA/ALU pipes (offloads the SFU): x = n + f with
// n = round(x) (magic-number rounding) and f in [-1/2, 1/2]; 2^f by a cubic
// fitted to 2^f on [-1/2, 1/2] with p(0) = 1 (iteratively reweighted least
// squares on the relative error; max relative error 1.0e-4); 2^n is added to
// the exponent field.  Inputs below -126 (masked scores) give ~2^-126.
PM_DEVICE float exp2_poly(float x) {
  x = fmaxf(x, -126.0f);
  const float t = x + 12582912.0f;  // 1.5 * 2^23: round(x) in the low mantissa bits
  const float f = x - (t - 12582912.0f);
  const float p = fmaf(fmaf(fmaf(0.05500864f, f, 0.2422105f), f, 0.69328291f), f, 1.0f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// Forward with two query tiles per CTA: tile 0 = queries [q0, q0+128), tile 1 =
// [q0+128, q0+256) of one (batch, head).  320 threads:
//   warp 0      TMA: Q0, Q1 once; K_j / V_j through a 3-slot ring
//   warp 1      MMA, one lane: S0_0, S1_0, then per key tile j:
//               O0 += P0_j V_j, S0_{j+1}, O1 += P1_j V_j, S1_{j+1}
//               so each softmax group works while the other tile's MMAs run
//   warps 2-5   softmax of tile 0, warps 6-9 softmax of tile 1 (one row per
//               thread): pass 1 reads the S row from TMEM for the row max, pass
//               2 reads it again and writes P (bf16, swizzled smem).  The
//               exponent base moves only when the row max grows by more than 8
//               (log2 units), so O is rarely rescaled; about a quarter of the
//               exponentials run as a polynomial on the FMA pipe.
//   TMEM: S0 | S1 | O0 | O1 (512 columns).
constexpr int kFwd2Threads = 320;
constexpr int kPolyPer32 = 8;  // exponentials per 32 evaluated by exp2_poly

// Row max of the raw scores of one 128-key S row in TMEM (keys outside [lo, hi] masked when MASK).
template <bool MASK>
PM_DEVICE float srow_max(uint32_t t_s, int lo, int hi) {
  float mraw = -INFINITY;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t v0[32], v1[32];
    tmem_ld32(t_s + half * 64, v0);
    tmem_ld32(t_s + half * 64 + 32, v1);
    tmem_ld_wait();
    if (MASK) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (half * 64 + i > hi || half * 64 + i < lo) v0[i] = __float_as_uint(-INFINITY);
        if (half * 64 + 32 + i > hi || half * 64 + 32 + i < lo) v1[i] = __float_as_uint(-INFINITY);
      }
    }
#pragma unroll
    for (int i = 0; i < 32; i += 2)
      mraw = max3f(mraw, max3f(__uint_as_float(v0[i]), __uint_as_float(v0[i + 1]), __uint_as_float(v1[i])),
                   __uint_as_float(v1[i + 1]));
  }
  return mraw;
}

// P = 2^(s c - m) of one S row -> bf16 into the swizzled P buffer (keys outside [lo, hi]
// masked when MASK); returns the row sum.
template <bool MASK>
PM_DEVICE float srow_exp_store(uint32_t t_s, int r, int lo, int hi, float c, float m, uint8_t* myP) {
  const uint64_t c2 = f2_pack(c, c), nm2 = f2_pack(-m, -m);
  uint64_t sum2 = f2_pack(0.f, 0.f);
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    uint32_t v[32];
    tmem_ld32(t_s + cc * 32, v);
    tmem_ld_wait();
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      float x0, x1;
      f2_unpack(fma_f2(f2_pack(__uint_as_float(v[i]), __uint_as_float(v[i + 1])), c2, nm2), x0, x1);
      if (MASK) {
        if (cc * 32 + i > hi || cc * 32 + i < lo) x0 = -INFINITY;
        if (cc * 32 + i + 1 > hi || cc * 32 + i + 1 < lo) x1 = -INFINITY;
      }
      const float p0 = ((i >> 1) % (16 / kPolyPer32) == 0) ? exp2_poly(x0) : fast_exp2(x0);
      const float p1 = fast_exp2(x1);
      sum2 = add_f2(sum2, f2_pack(p0, p1));
      pk[i >> 1] = pack_bf16(p0, p1);
    }
#pragma unroll
    for (int q8 = 0; q8 < 4; ++q8) {
      const int chunk = cc * 4 + q8;  // 16-byte chunk of the 128-key row
      st_swz(myP + (chunk >> 3) * 16384, r, chunk & 7,
             make_uint4(pk[4 * q8], pk[4 * q8 + 1], pk[4 * q8 + 2], pk[4 * q8 + 3]));
    }
  }
  float s0, s1;
  f2_unpack(sum2, s0, s1);
  return s0 + s1;
}

template <int D>
__global__ void __launch_bounds__(kFwd2Threads, 1)
    attn_fwd2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, AttnArgs a) {
  constexpr int ND = D / 64;
  constexpr int kTB = ND * 16384;  // one [128 x D] bf16 tile
  constexpr int kSlots = 3;
  constexpr uint32_t kIdescS = make_idesc_bf16(128, 128, false, false);
  constexpr uint32_t kIdescO = make_idesc_bf16(128, D, false, true);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sQ = sm;                     // 2 tiles
  uint8_t* sKV = sQ + 2 * kTB;          // kSlots tiles
  uint8_t* sP = sKV + kSlots * kTB;     // 2 x 32 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * 32768);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;              // [kSlots]
  uint64_t* kv_empty = bars + 1 + kSlots;    // [kSlots]
  uint64_t* s_full = bars + 1 + 2 * kSlots;  // [2]
  uint64_t* p_full = s_full + 2;             // [2]
  uint64_t* pv_done = p_full + 2;            // [2]
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(pv_done + 2);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int npairs = a.S / 256;
  const int L = blockIdx.x;
  const int pt = npairs - 1 - L / (a.B * a.Hq);  // heaviest tiles first
  const int rem = L % (a.B * a.Hq);
  const int b = rem / a.Hq, h = rem % a.Hq;
  const int hk = h / (a.Hq / a.Hkv);
  const int qa = 2 * pt;  // key-tile index of tile 0's diagonal
  const int tq0 = b * a.S + qa * kTile;
  const int n0 = qa + 1, n1 = qa + 2;  // key tiles seen by tile 0 / tile 1

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kSlots; ++i) { mbar_init(&kv_full[i], 1); mbar_init(&kv_empty[i], 1); }
    for (int g = 0; g < 2; ++g) { mbar_init(&s_full[g], 1); mbar_init(&p_full[g], 128); mbar_init(&pv_done[g], 1); }
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) { tmem_alloc(s_tmem, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 2 * kTB);
#pragma unroll
      for (int g = 0; g < 2; ++g)
#pragma unroll
        for (int d = 0; d < ND; ++d) tma_load_3d(sQ + g * kTB + d * 16384, &tmQ, q_full, d * 64, h, tq0 + g * kTile);
      // ring use u: K_j = 2j, V_j = 2j + 1
      for (int u = 0; u < 2 * n1; ++u) {
        const int slot = u % kSlots;
        if (!mbar_wait_abortable(&kv_empty[slot], ((u / kSlots) & 1) ^ 1, s_abort)) break;
        const int tk0 = b * a.S + (u >> 1) * kTile;
        mbar_arrive_expect_tx(&kv_full[slot], kTB);
        const CUtensorMap* tm = (u & 1) ? &tmV : &tmK;
#pragma unroll
        for (int d = 0; d < ND; ++d) tma_load_3d(sKV + slot * kTB + d * 16384, tm, &kv_full[slot], d * 64, hk, tk0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t aq0 = smem_u32(sQ), aq1 = smem_u32(sQ + kTB);
      const uint32_t ap0 = smem_u32(sP), ap1 = smem_u32(sP + 32768);
      auto kv_wait = [&](int u) { return mbar_wait_abortable(&kv_full[u % kSlots], (u / kSlots) & 1, s_abort); };
      auto s_mma = [&](int g, int u) {
        const uint32_t ak = smem_u32(sKV + (u % kSlots) * kTB);
        const uint32_t aq = g ? aq1 : aq0;
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          umma_f16(tmem + g * 128, kmaj_desc(aq, k), kmaj_desc(ak, k), kIdescS, k > 0);
        umma_commit(&s_full[g]);
      };
      auto pv_mma = [&](int g, int u, bool first) {
        const uint32_t av = smem_u32(sKV + (u % kSlots) * kTB);
        const uint32_t ap = g ? ap1 : ap0;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_f16(tmem + 256 + g * D, kmaj_desc(ap, k), mnmaj_desc(av, k), kIdescO, (!first || k > 0));
        umma_commit(&pv_done[g]);
      };
      bool ok = mbar_wait_abortable(q_full, 0, s_abort) && kv_wait(0);
      if (ok) {
        tc_fence_after();
        s_mma(0, 0);
        s_mma(1, 0);
        umma_commit(&kv_empty[0]);
      }
      for (int j = 0; ok && j < n1; ++j) {
        const int uk = 2 * (j + 1), uv = 2 * j + 1;
        bool k_ready = false;
        if (j < n0) {
          ok = mbar_wait_abortable(&p_full[0], j & 1, s_abort) && kv_wait(uv);
          if (!ok) break;
          tc_fence_after();
          pv_mma(0, uv, j == 0);
          if (j + 1 < n0) {
            if (!(ok = kv_wait(uk))) break;
            k_ready = true;
            tc_fence_after();
            s_mma(0, uk);
          }
        }
        ok = mbar_wait_abortable(&p_full[1], j & 1, s_abort) && kv_wait(uv);
        if (!ok) break;
        tc_fence_after();
        pv_mma(1, uv, j == 0);
        umma_commit(&kv_empty[uv % kSlots]);
        if (j + 1 < n1) {
          if (!k_ready && !(ok = kv_wait(uk))) break;
          tc_fence_after();
          s_mma(1, uk);
          umma_commit(&kv_empty[uk % kSlots]);
        }
      }
      if (!ok) *s_abort = 1;
    }
  } else {
    // softmax: tile g, one query row per thread
    const int g = (warp - 2) >> 2;
    const int qd = warp & 3;
    const int r = qd * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(qd * 32) << 16);
    const uint32_t t_s = trow + g * 128, t_o = trow + 256 + g * D;
    uint8_t* myP = sP + g * 32768;
    const int ng = g ? n1 : n0;
    const int diag = qa + g;
    const float c = a.scale * kLog2e;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    // first key of this row's document (packed sequences); 0 = the whole causal prefix
    const int qlo = a.doc_lo ? a.doc_lo[tq0 + g * kTile + r] : 0;
    for (int j = 0; j < ng; ++j) {
      if (!mbar_wait_abortable(&s_full[g], j & 1, s_abort)) { ok = false; break; }
      tc_fence_after();
      const int lo = qlo - j * kTile, hi = j == diag ? r : kTile - 1;
      // warp-uniform choice: the row helpers issue warp-collective TMEM loads (a fully masked row
      // keeps m = -inf and adds 0; rows without masking have lo <= 0 and hi = 127)
      const bool masked = __any_sync(0xffffffffu, j == diag || lo > 0);
      // pass 1: row max (raw scores; the scale is positive)
      const float mraw = masked ? srow_max<true>(t_s, lo, hi) : srow_max<false>(t_s, 0, kTile - 1);
      const float mx = mraw * c;
      float alpha = 1.0f;
      if (mx > m + 8.0f) {  // move the exponent base only when the max grew a lot
        alpha = fast_exp2(m - mx);  // 0 on the first tile
        m = mx;
      }
      l *= alpha;
      if (j > 0) {
        // P buffer free and O complete for key tile j - 1
        if (!mbar_wait_abortable(&pv_done[g], (j - 1) & 1, s_abort)) { ok = false; break; }
        tc_fence_after();
        if (!__all_sync(0xffffffffu, alpha == 1.0f)) {
          const uint64_t a2 = f2_pack(alpha, alpha);
#pragma unroll
          for (int cc = 0; cc < D / 16; ++cc) {
            uint32_t v[16];
            tmem_ld16(t_o + cc * 16, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
              float x0, x1;
              f2_unpack(mul_f2(f2_pack(__uint_as_float(v[i]), __uint_as_float(v[i + 1])), a2), x0, x1);
              v[i] = __float_as_uint(x0);
              v[i + 1] = __float_as_uint(x1);
            }
            tmem_st16(t_o + cc * 16, v);
          }
          tmem_st_wait();
        }
      }
      // pass 2: P = 2^(s c - m) -> bf16, swizzled into the A operand buffer
      l += masked ? srow_exp_store<true>(t_s, r, lo, hi, c, m, myP)
                  : srow_exp_store<false>(t_s, r, 0, kTile - 1, c, m, myP);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[g]);
    }
    if (ok && mbar_wait_abortable(&pv_done[g], (ng - 1) & 1, s_abort)) {
      tc_fence_after();
      const float inv = 1.f / l;
      __nv_bfloat16* orow = a.o + ((size_t)(tq0 + g * kTile + r) * a.Hq + h) * D;
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t v[32];
        tmem_ld32(t_o + cc * 32, v);
        tmem_ld_wait();
        uint4* dst = reinterpret_cast<uint4*>(orow + cc * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          dst[i] = make_uint4(pack_bf16(__uint_as_float(v[8 * i]) * inv, __uint_as_float(v[8 * i + 1]) * inv),
                              pack_bf16(__uint_as_float(v[8 * i + 2]) * inv, __uint_as_float(v[8 * i + 3]) * inv),
                              pack_bf16(__uint_as_float(v[8 * i + 4]) * inv, __uint_as_float(v[8 * i + 5]) * inv),
                              pack_bf16(__uint_as_float(v[8 * i + 6]) * inv, __uint_as_float(v[8 * i + 7]) * inv));
      }
      a.lse[(size_t)h * a.T + tq0 + g * kTile + r] = (m + __log2f(l)) * kLn2;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D>
constexpr int fwd2_smem() {
  return (2 + 3) * (D / 64) * 16384 + 2 * 32768 + 1024 + 256;
}

// delta[h, t] = sum_d dO[t, h, d] * O[t, h, d]
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout, int T,
                                  int Hq, int D, float* __restrict__ delta) {
  const int w = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (w >= T * Hq) return;
  const int t = w / Hq, h = w % Hq;
  const __nv_bfloat16* po = o + (size_t)w * D;
  const __nv_bfloat16* pd = dout + (size_t)w * D;
  float s = 0.f;
  for (int i = lane * 2; i < D; i += 64) {
    const __nv_bfloat162 x = *reinterpret_cast<const __nv_bfloat162*>(po + i);
    const __nv_bfloat162 y = *reinterpret_cast<const __nv_bfloat162*>(pd + i);
    s += __low2float(x) * __low2float(y) + __high2float(x) * __high2float(y);
  }
  s = warp_sum(s);
  if (lane == 0) delta[(size_t)h * T + t] = s;
}

// ---------------------------------------------------------------- backward
// One CTA per (batch, kv head, 128-key tile), 320 threads; iterations i run over
// the q heads of the GQA group and the q tiles at or after the key tile.
//   warp 0      TMA: K, V once; Q_i (+ its LSE and delta rows) through two stages,
//               dO_i through one stage.
//   warp 1      MMA, one lane, in this order per iteration:
//                 dP_i^T = V dO_i^T               -> TMEM B
//                 dV    += P_i^T dO_i              (A operand = P^T read from TMEM A)
//                 S_{i+1}^T = K Q_{i+1}^T         -> TMEM A (after dV_i has read P_i^T)
//                 dK    += dS_i^T Q_i              (dS^T from shared memory)
//                 dQ_i   = dS_i K                 -> TMEM B (dP_i^T was consumed)
//               so the tensor pipe only waits while dQ_i is read out of TMEM.
//   warps 2-9   two warpgroups; warp w owns TMEM lane quarter w % 4 (32 key rows, or
//               32 query rows of dQ) and column group (w - 2) / 4 (64 queries, D / 2
//               head dims), with packed f32x2 arithmetic:
//               per tile i: dS_i^T = P_i^T (dP_i^T - delta) scale to swizzled shared memory
//               (P_i kept in registers as bf16 pairs), then P_{i+1}^T = 2^(S^T c - lse)
//               written bf16 into its own S^T columns (TMEM) while dK_i / dQ_i run,
//               dQ_i read from TMEM into fp32 staging boxes [128 queries x 32 dims]
//               (128B-swizzled) that one thread per warpgroup adds to the fp32 dQ
//               buffer with TMA reduce-adds.  Boxes 0-1 have their own 32 KB; boxes
//               2-3 (D = 128) reuse the dS^T buffer, free once dQ_i completed, and
//               dS_{i+1} is written only after those reductions finished reading it.
//   TMEM: A = S^T / P^T (128 cols) | B = dP^T / dQ (128) | dV (D) | dK (D).
// P^T of queries [64g, 64g + 64) sits in columns [64g, 64g + 32) of A (two bf16 per
// column), so each MMA k-step of 16 queries reads 8 columns.
// CTAs run (batch, kv head) outer and key tile inner, so the CTAs resident at one time
// share a few heads and their Q / dO tiles and dQ reductions stay in L2.
constexpr int kBwdThreads = 320;
constexpr int kBwdCompute = 256;  // threads of the two compute warpgroups

// K, V, two Q stages, dO, dS^T, dQ staging (32 KB), LSE / delta stages, barriers.  The
// base of dynamic shared memory must be 1024-byte aligned (checked in the kernel).
template <int D>
constexpr int bwd_smem() {
  return 5 * (D / 64) * 16384 + 32768 + 32768 + 2048 + 128;
}

// P = 2^(S c - lse) for 32 queries of one key row, as bf16 pairs.  When MASK, query columns
// outside [rel, rhi) are masked: rel = key - first query (causal), rhi = end of the key's
// document - first query (packed sequences).
template <bool MASK>
PM_DEVICE void bwd_probs(const uint32_t (&sv)[32], const float4* lse4, float c, int rel, int rhi, uint32_t* pk) {
  const uint64_t c2 = f2_pack(c, c);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 l = lse4[j];
    const uint64_t x0 = fma_f2(f2_pack(__uint_as_float(sv[4 * j]), __uint_as_float(sv[4 * j + 1])), c2,
                               f2_pack(-l.x, -l.y));
    const uint64_t x1 = fma_f2(f2_pack(__uint_as_float(sv[4 * j + 2]), __uint_as_float(sv[4 * j + 3])), c2,
                               f2_pack(-l.z, -l.w));
    float e[4];
    f2_unpack(x0, e[0], e[1]);
    f2_unpack(x1, e[2], e[3]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      e[k] = fast_exp2(e[k]);
      if (MASK && (4 * j + k < rel || 4 * j + k >= rhi)) e[k] = 0.f;
    }
    pk[2 * j] = pack_bf16(e[0], e[1]);
    pk[2 * j + 1] = pack_bf16(e[2], e[3]);
  }
}

template <int D>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    const __grid_constant__ CUtensorMap tmDQ, AttnArgs a) {
  constexpr int ND = D / 64;
  constexpr int kTB = ND * 16384;  // one [128 x D] bf16 tile
  constexpr int kQD = D / 2;       // head dims per compute thread (dQ, dK, dV)
  constexpr int kBoxes = kQD / 32;  // dQ staging boxes per warpgroup
  constexpr bool kBoxesInDS = D == 128;  // boxes 2-3 (warpgroup 1) are staged in the dS^T buffer
  constexpr uint32_t kIdescS = make_idesc_bf16(128, 128, false, false);  // S^T, dP^T
  constexpr uint32_t kIdescKV = make_idesc_bf16(128, D, false, true);   // dV, dK
  constexpr uint32_t kIdescQ = make_idesc_bf16(128, D, true, true);     // dQ (A = dS, MN-major)

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023u) {  // swizzled tiles need 1024-byte alignment: refuse, do not misread
    if (threadIdx.x == 0) set_error(kErrArgs);
    return;
  }
  uint8_t* sK = smem_raw;
  uint8_t* sV = sK + kTB;
  uint8_t* sQ0 = sV + kTB;        // two Q stages
  uint8_t* sDO = sQ0 + 2 * kTB;
  uint8_t* sDS = sDO + kTB;       // 32 KB: dS^T [keys x queries]
  uint8_t* sStage = sDS + 32768;  // 32 KB: dQ staging boxes 0-1
  float* sLse = reinterpret_cast<float*>(sStage + 32768);  // [2][128], log2 units
  float* sDelta = sLse + 256;                               // [2][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDelta + 256);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;   // [2]
  uint64_t* q_empty = bars + 3;  // [2]
  uint64_t* do_full = bars + 5;
  uint64_t* do_empty = bars + 6;
  uint64_t* s_full = bars + 7;
  uint64_t* dp_full = bars + 8;
  uint64_t* dq_full = bars + 9;
  uint64_t* p_done = bars + 10;
  uint64_t* ds_done = bars + 11;
  uint64_t* dq_drained = bars + 12;
  uint64_t* dkv_full = bars + 13;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = a.S / kTile;
  const int G = a.Hq / a.Hkv;
  const int L = blockIdx.x;
  const int kt = L % nq;  // within a head, the key tiles with the most q tiles start first
  const int rem = L / nq;
  const int b = rem / a.Hkv, hk = rem % a.Hkv;
  const int tk0 = b * a.S + kt * kTile;
  const int nqt = nq - kt;
  const int n_it = G * nqt;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(&q_full[0], 1); mbar_init(&q_full[1], 1);
    mbar_init(&q_empty[0], 1); mbar_init(&q_empty[1], 1);
    mbar_init(do_full, 1); mbar_init(do_empty, 1);
    mbar_init(s_full, 1); mbar_init(dp_full, 1); mbar_init(dq_full, 1);
    mbar_init(p_done, kBwdCompute); mbar_init(ds_done, kBwdCompute); mbar_init(dq_drained, kBwdCompute);
    mbar_init(dkv_full, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) { tmem_alloc(s_tmem, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const uint32_t tA = tmem, tB = tmem + 128, tDV = tmem + 256, tDK = tmem + 256 + D;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * kTB);
#pragma unroll
      for (int d = 0; d < ND; ++d) {
        tma_load_3d(sK + d * 16384, &tmK, kv_full, d * 64, hk, tk0);
        tma_load_3d(sV + d * 16384, &tmV, kv_full, d * 64, hk, tk0);
      }
      for (int it = 0; it < n_it; ++it) {
        const int h = hk * G + it / nqt;
        const int tq0 = b * a.S + (kt + it % nqt) * kTile;
        const int st = it & 1;
        if (!mbar_wait_abortable(&q_empty[st], ((it >> 1) & 1) ^ 1, s_abort)) break;
        mbar_arrive_expect_tx(&q_full[st], kTB + 1024);
#pragma unroll
        for (int d = 0; d < ND; ++d) tma_load_3d(sQ0 + st * kTB + d * 16384, &tmQ, &q_full[st], d * 64, h, tq0);
        bulk_load(sLse + st * 128, a.lse_in + (size_t)h * a.T + tq0, 512, &q_full[st]);
        bulk_load(sDelta + st * 128, a.delta + (size_t)h * a.T + tq0, 512, &q_full[st]);
        if (!mbar_wait_abortable(do_empty, (it & 1) ^ 1, s_abort)) break;
        mbar_arrive_expect_tx(do_full, kTB);
#pragma unroll
        for (int d = 0; d < ND; ++d) tma_load_3d(sDO + d * 16384, &tmDO, do_full, d * 64, h, tq0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), aDO = smem_u32(sDO), aDS = smem_u32(sDS);
      const uint32_t aQ0 = smem_u32(sQ0);
      bool ok = mbar_wait_abortable(kv_full, 0, s_abort) && mbar_wait_abortable(&q_full[0], 0, s_abort);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < D / 16; ++k) umma_f16(tA, kmaj_desc(aK, k), kmaj_desc(aQ0, k), kIdescS, k > 0);
        umma_commit(s_full);
      }
      for (int it = 0; ok && it < n_it; ++it) {
        const uint32_t aQ = aQ0 + (it & 1) * kTB;
        // dP_i^T -> B once dO_i landed and dQ_{i-1} left B
        if (!mbar_wait_abortable(do_full, it & 1, s_abort)) break;
        if (it > 0 && !mbar_wait_abortable(dq_drained, (it - 1) & 1, s_abort)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < D / 16; ++k) umma_f16(tB, kmaj_desc(aV, k), kmaj_desc(aDO, k), kIdescS, k > 0);
        umma_commit(dp_full);
        // dV += P_i^T dO_i with P^T from TMEM
        if (!mbar_wait_abortable(p_done, it & 1, s_abort)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_f16_ts(tDV, tA + (k >> 2) * 64 + (k & 3) * 8, mnmaj_desc(aDO, k), kIdescKV, (it > 0 || k > 0));
        umma_commit(do_empty);
        // S_{i+1}^T -> A (ordered after dV_i, which read P_i^T from A)
        if (it + 1 < n_it) {
          if (!mbar_wait_abortable(&q_full[(it + 1) & 1], ((it + 1) >> 1) & 1, s_abort)) break;
          tc_fence_after();
          const uint32_t aQn = aQ0 + ((it + 1) & 1) * kTB;
#pragma unroll
          for (int k = 0; k < D / 16; ++k) umma_f16(tA, kmaj_desc(aK, k), kmaj_desc(aQn, k), kIdescS, k > 0);
          umma_commit(s_full);
        }
        // dK += dS_i^T Q_i, dQ_i = dS_i K -> B
        if (!mbar_wait_abortable(ds_done, it & 1, s_abort)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) umma_f16(tDK, kmaj_desc(aDS, k), mnmaj_desc(aQ, k), kIdescKV, (it > 0 || k > 0));
        umma_commit(&q_empty[it & 1]);
#pragma unroll
        for (int k = 0; k < 8; ++k) umma_f16(tB, mnmaj_desc(aDS, k), mnmaj_desc(aK, k), kIdescQ, k > 0);
        umma_commit(dq_full);
      }
      umma_commit(dkv_full);  // also on abort: every issued MMA completes before TMEM is freed
    }
  } else {
    const int qd = warp & 3;
    const int cg = (warp - 2) >> 2;
    const int r = qd * 32 + lane;  // key row (S^T, dP^T, dV, dK) / query row (dQ)
    const uint32_t lrow = (uint32_t)(qd * 32) << 16;
    const float c = a.scale * kLog2e;
    // dQ staging: a box holds 32 head dims of all 128 queries; warpgroup cg owns boxes
    // kBoxes * cg ...; boxes 0-1 live in the staging buffer, 2-3 in the dS^T buffer
    uint8_t* bx0 = cg == 0 ? sStage : (kBoxesInDS ? sDS : sStage + 16384);
    const bool issuer = qd == 0 && lane == 0;
    // A failed (bounded) wait only skips work: every thread still reaches the named barriers,
    // and the decision to stop is taken uniformly by all compute threads (bar.red.and).
    bool ok = true;
    // P of tile j (64 queries of this group, bf16 pairs) -> TMEM (A operand of dV) and `pk`
    // (kept for dS, since the next S^T MMA overwrites the TMEM copy).
    uint32_t pk[32];
    // end of this key's document (packed sequences), relative to the row of seq_len tokens
    const int khi = a.doc_hi ? a.doc_hi[tk0 + r] : a.S;
    auto probs = [&](int j) {
      const int st = j & 1;
      const int qt_j = kt + j % nqt;
      const bool diag = qt_j == kt;
      ok = ok && mbar_wait_abortable(&q_full[st], (j >> 1) & 1, s_abort) &&  // LSE rows visible
           mbar_wait_abortable(s_full, j & 1, s_abort);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) return;
      tc_fence_after();
      const float4* lse4 = reinterpret_cast<const float4*>(sLse + st * 128 + cg * 64);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t sv[32];
        const int q0 = cg * 64 + half * 32;
        tmem_ld32(tA + lrow + q0, sv);
        tmem_ld_wait();
        const int rhi = khi - (qt_j * kTile + q0);
        if (diag || rhi < 32) bwd_probs<true>(sv, lse4 + half * 8, c, diag ? r - q0 : 0, rhi, pk + half * 16);
        else bwd_probs<false>(sv, lse4 + half * 8, c, 0, 32, pk + half * 16);
        // P^T bf16 over the group's own S^T columns (already read)
        tmem_st16(tA + lrow + cg * 64 + half * 16, *reinterpret_cast<uint32_t(*)[16]>(pk + half * 16));
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_done);
    };
    probs(0);
    const uint64_t sc2 = f2_pack(a.scale, a.scale);
    for (int it = 0; it < n_it; ++it) {
      const int h = hk * G + it / nqt;
      const int qt = kt + it % nqt;
      const int tq0 = b * a.S + qt * kTile;
      const int st = it & 1;
      const float4* dl4 = reinterpret_cast<const float4*>(sDelta + st * 128 + cg * 64);
      // dS^T = P^T (dP^T - delta) * scale -> swizzled shared memory
      ok = ok && mbar_wait_abortable(dp_full, it & 1, s_abort);
      ok = __all_sync(0xffffffffu, ok);
      if constexpr (kBoxesInDS) {
        // the dQ reductions of the previous tile read staging boxes 2-3 out of the dS^T buffer
        if (issuer && cg == 1) bulk_wait_read_0();
        ok = named_bar_and(5, kBwdCompute, ok);
      }
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t pv[32], dsk[16];
          tmem_ld32(tB + lrow + cg * 64 + half * 32, pv);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 d = dl4[half * 8 + j];
            const uint32_t p01 = pk[half * 16 + 2 * j], p23 = pk[half * 16 + 2 * j + 1];
            const uint64_t t0 = add_f2(f2_pack(__uint_as_float(pv[4 * j]), __uint_as_float(pv[4 * j + 1])),
                                       f2_pack(-d.x, -d.y));
            const uint64_t t1 = add_f2(f2_pack(__uint_as_float(pv[4 * j + 2]), __uint_as_float(pv[4 * j + 3])),
                                       f2_pack(-d.z, -d.w));
            float u0, u1, u2, u3;
            f2_unpack(mul_f2(mul_f2(f2_pack(bf16_lo(p01), bf16_hi(p01)), sc2), t0), u0, u1);
            f2_unpack(mul_f2(mul_f2(f2_pack(bf16_lo(p23), bf16_hi(p23)), sc2), t1), u2, u3);
            dsk[2 * j] = pack_bf16(u0, u1);
            dsk[2 * j + 1] = pack_bf16(u2, u3);
          }
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int chunk = cg * 8 + half * 4 + g;  // 8 queries per 16-byte chunk
            st_swz(sDS + (chunk >> 3) * 16384, r, chunk & 7,
                   make_uint4(dsk[4 * g], dsk[4 * g + 1], dsk[4 * g + 2], dsk[4 * g + 3]));
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(ds_done);
      }
      // P of the next tile while the tensor pipe runs dK_i and dQ_i (S_{i+1} was issued after dV_i)
      if (it + 1 < n_it) probs(it + 1);
      // dQ_i (rows = queries): TMEM -> registers (B released) -> staging boxes -> TMA reduce-add
      ok = ok && mbar_wait_abortable(dq_full, it & 1, s_abort);
      ok = __all_sync(0xffffffffu, ok);
      uint32_t dq[kQD];
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < kBoxes; ++cc) {
          uint32_t (&v)[32] = *reinterpret_cast<uint32_t(*)[32]>(dq + cc * 32);
          tmem_ld32(tB + lrow + cg * kQD + cc * 32, v);
        }
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(dq_drained);
      }
      if (issuer) bulk_wait_read_0();  // this group's previous reductions have read its staging
      if (!named_bar_and(6, kBwdCompute, ok)) { ok = false; break; }
#pragma unroll
      for (int cc = 0; cc < kBoxes; ++cc)
#pragma unroll
        for (int i = 0; i < 8; ++i)
          st_swz(bx0 + cc * 16384, r, i,
                 make_uint4(dq[cc * 32 + 4 * i], dq[cc * 32 + 4 * i + 1], dq[cc * 32 + 4 * i + 2],
                            dq[cc * 32 + 4 * i + 3]));
      fence_proxy_async_smem();
      named_bar_sync(1 + cg, 128);
      if (issuer) {
#pragma unroll
        for (int cc = 0; cc < kBoxes; ++cc) tma_reduce_add_3d(&tmDQ, bx0 + cc * 16384, cg * kQD + cc * 32, h, tq0);
        bulk_commit();
      }
    }
    if (issuer) bulk_wait_all();  // reductions complete before the CTA's shared memory goes away
    if (ok && mbar_wait_abortable(dkv_full, 0, s_abort)) {
      tc_fence_after();
#pragma unroll 1
      for (int cc = 0; cc < kQD / 32; ++cc) {
        uint32_t v[32], w[32];
        tmem_ld32(tDV + lrow + cg * kQD + cc * 32, v);
        tmem_ld32(tDK + lrow + cg * kQD + cc * 32, w);
        tmem_ld_wait();
        uint4* dv4 = reinterpret_cast<uint4*>(a.dv + ((size_t)(tk0 + r) * a.Hkv + hk) * D + cg * kQD + cc * 32);
        uint4* dk4 = reinterpret_cast<uint4*>(a.dk + ((size_t)(tk0 + r) * a.Hkv + hk) * D + cg * kQD + cc * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          dv4[i] = make_uint4(pack_bf16(__uint_as_float(v[8 * i]), __uint_as_float(v[8 * i + 1])),
                              pack_bf16(__uint_as_float(v[8 * i + 2]), __uint_as_float(v[8 * i + 3])),
                              pack_bf16(__uint_as_float(v[8 * i + 4]), __uint_as_float(v[8 * i + 5])),
                              pack_bf16(__uint_as_float(v[8 * i + 6]), __uint_as_float(v[8 * i + 7])));
          dk4[i] = make_uint4(pack_bf16(__uint_as_float(w[8 * i]), __uint_as_float(w[8 * i + 1])),
                              pack_bf16(__uint_as_float(w[8 * i + 2]), __uint_as_float(w[8 * i + 3])),
                              pack_bf16(__uint_as_float(w[8 * i + 4]), __uint_as_float(w[8 * i + 5])),
                              pack_bf16(__uint_as_float(w[8 * i + 6]), __uint_as_float(w[8 * i + 7])));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    // every MMA this CTA issued has completed once dkv_full fired (bounded wait)
    mbar_wait(dkv_full, 0);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// fp32 -> bf16
__global__ void f32_to_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, long long n) {
  const long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i + 3 < n) {
    const float4 v = *reinterpret_cast<const float4*>(src + i);
    *reinterpret_cast<uint2*>(dst + i) = make_uint2(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w));
  } else {
    for (long long j = i; j < n; ++j) dst[j] = __float2bfloat16(src[j]);
  }
}

// ------------------------------------------------------------------ host
static CUtensorMap head_map(const torch::Tensor& t) {
  // t: [T, H, D] contiguous bf16 -> dims {D, H, T}, box {64, 1, 128}
  const int64_t T = t.size(0), H = t.size(1), D = t.size(2);
  CUtensorMap m;
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T};
  cuuint64_t strides[2] = {(cuuint64_t)(D * 2), (cuuint64_t)(H * D * 2)};
  cuuint32_t box[3] = {64, 1, 128};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_tiled_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, t.data_ptr(), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "attention tensor map failed: ", (int)r);
  return m;
}

// fp32 dQ accumulator [T, Hq, D] -> dims {D, Hq, T}, box {32, 1, 128}, 128B swizzle (reduce-add target)
static CUtensorMap dq_acc_map(const torch::Tensor& t) {
  const int64_t T = t.size(0), H = t.size(1), D = t.size(2);
  CUtensorMap m;
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T};
  cuuint64_t strides[2] = {(cuuint64_t)(D * 4), (cuuint64_t)(H * D * 4)};
  cuuint32_t box[3] = {32, 1, 128};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_tiled_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, t.data_ptr(), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "dQ tensor map failed: ", (int)r);
  return m;
}

static void check_qkv(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, int64_t S) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == torch::kBFloat16 && q.is_contiguous() && q.dim() == 3, "q [T,Hq,D] bf16");
  TORCH_CHECK(k.sizes() == v.sizes() && k.is_contiguous() && v.is_contiguous(), "k/v layout");
  PM_CHECK_CUDA(k); PM_CHECK_CUDA(v);
  TORCH_CHECK(k.scalar_type() == torch::kBFloat16 && v.scalar_type() == torch::kBFloat16, "k/v bf16");
  TORCH_CHECK(k.size(0) == q.size(0) && k.size(2) == q.size(2), "k/v shape");
  TORCH_CHECK(q.size(1) % k.size(1) == 0, "Hq must be a multiple of Hkv");
  TORCH_CHECK(S % kTile == 0 && q.size(0) % S == 0, "seq_len must be a multiple of 128 and divide T");
  TORCH_CHECK(q.size(2) == 64 || q.size(2) == 128, "head_dim must be 64 or 128");
}

template <int D>
static int fwd_smem() { return 1024 + (5 * (D / 64) * 16384) + 32768 + 256; }

// Per-token int32 positions of packed documents (see AttnArgs::doc_lo / doc_hi).
static const int* doc_ptr(const c10::optional<torch::Tensor>& t, const torch::Tensor& q, const char* name) {
  if (!t.has_value()) return nullptr;
  TORCH_CHECK(t->is_cuda() && t->device() == q.device() && t->scalar_type() == torch::kInt32 &&
                  t->is_contiguous() && t->numel() == q.size(0),
              name, " must be a contiguous int32 CUDA tensor with one entry per token");
  return t->data_ptr<int>();
}

std::vector<torch::Tensor> attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, int64_t S,
                                    c10::optional<torch::Tensor> doc_lo) {
  check_qkv(q, k, v, S);
  TORCH_CHECK(!doc_lo.has_value() || S % 256 == 0, "packed documents need seq_len % 256 == 0");
  c10::cuda::CUDAGuard guard(q.device());
  const int T = (int)q.size(0), Hq = (int)q.size(1), Hkv = (int)k.size(1), D = (int)q.size(2);
  auto o = torch::empty_like(q);
  auto lse = torch::empty({Hq, T}, q.options().dtype(torch::kFloat32));
  if (T == 0) return {o, lse};
  AttnArgs a;
  memset(&a, 0, sizeof(a));
  a.T = T; a.S = (int)S; a.Hq = Hq; a.Hkv = Hkv; a.B = T / (int)S;
  a.scale = 1.f / sqrtf((float)D);
  a.o = (__nv_bfloat16*)o.data_ptr();
  a.lse = lse.data_ptr<float>();
  a.doc_lo = doc_ptr(doc_lo, q, "doc_lo");
  CUtensorMap mq = head_map(q), mk = head_map(k), mv = head_map(v);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (S % 256 == 0) {  // two query tiles per CTA
    const int grid2 = a.B * Hq * ((int)S / 256);
    if (D == 128) {
      auto kern = attn_fwd2_kernel<128>;
      C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, fwd2_smem<128>()));
      kern<<<grid2, kFwd2Threads, fwd2_smem<128>(), stream>>>(mq, mk, mv, a);
    } else {
      auto kern = attn_fwd2_kernel<64>;
      C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, fwd2_smem<64>()));
      kern<<<grid2, kFwd2Threads, fwd2_smem<64>(), stream>>>(mq, mk, mv, a);
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return {o, lse};
  }
  const int grid = a.B * Hq * ((int)S / kTile);
  if (D == 128) {
    auto kern = attn_fwd_kernel<128>;
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, fwd_smem<128>()));
    kern<<<grid, kAttnThreads, fwd_smem<128>(), stream>>>(mq, mk, mv, a);
  } else {
    auto kern = attn_fwd_kernel<64>;
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, fwd_smem<64>()));
    kern<<<grid, kAttnThreads, fwd_smem<64>(), stream>>>(mq, mk, mv, a);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {o, lse};
}

std::vector<torch::Tensor> attn_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o,
                                    torch::Tensor lse, torch::Tensor dout, int64_t S,
                                    c10::optional<torch::Tensor> doc_hi) {
  check_qkv(q, k, v, S);
  TORCH_CHECK(dout.is_contiguous() && dout.sizes() == q.sizes() && o.sizes() == q.sizes(), "dout / o layout");
  PM_CHECK_CUDA(o); PM_CHECK_CUDA(lse); PM_CHECK_CUDA(dout);
  TORCH_CHECK(lse.scalar_type() == torch::kFloat32 && lse.numel() == q.size(0) * q.size(1), "lse [Hq, T] fp32");
  c10::cuda::CUDAGuard guard(q.device());
  const int T = (int)q.size(0), Hq = (int)q.size(1), Hkv = (int)k.size(1), D = (int)q.size(2);
  auto dq = torch::empty_like(q);
  auto dk = torch::empty_like(k);
  auto dv = torch::empty_like(v);
  if (T == 0) return {dq, dk, dv};
  auto stream = at::cuda::getCurrentCUDAStream();
  auto delta = torch::empty({Hq, T}, q.options().dtype(torch::kFloat32));
  attn_delta_kernel<<<(T * Hq + 7) / 8, 256, 0, stream>>>((const __nv_bfloat16*)o.data_ptr(),
                                                          (const __nv_bfloat16*)dout.data_ptr(), T, Hq, D,
                                                          delta.data_ptr<float>());
  auto dq_acc = torch::zeros({T, Hq, D}, q.options().dtype(torch::kFloat32));
  AttnArgs a;
  memset(&a, 0, sizeof(a));
  a.T = T; a.S = (int)S; a.Hq = Hq; a.Hkv = Hkv; a.B = T / (int)S;
  a.scale = 1.f / sqrtf((float)D);
  a.delta = delta.data_ptr<float>();
  a.dq_acc = dq_acc.data_ptr<float>();
  a.dk = (__nv_bfloat16*)dk.data_ptr();
  a.dv = (__nv_bfloat16*)dv.data_ptr();
  a.doc_hi = doc_ptr(doc_hi, q, "doc_hi");
  // the kernel consumes the LSE in log2 units
  auto lse2 = (lse * kLog2e).contiguous();
  a.lse_in = lse2.data_ptr<float>();
  CUtensorMap mq = head_map(q), mk = head_map(k), mv = head_map(v), mdo = head_map(dout);
  CUtensorMap mdq = dq_acc_map(dq_acc);
  const int grid = a.B * Hkv * ((int)S / kTile);
  if (D == 128) {
    auto kern = attn_bwd_kernel<128>;
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bwd_smem<128>()));
    kern<<<grid, kBwdThreads, bwd_smem<128>(), stream>>>(mq, mk, mv, mdo, mdq, a);
  } else {
    auto kern = attn_bwd_kernel<64>;
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bwd_smem<64>()));
    kern<<<grid, kBwdThreads, bwd_smem<64>(), stream>>>(mq, mk, mv, mdo, mdq, a);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const long long n = (long long)T * Hq * D;
  f32_to_bf16_kernel<<<(unsigned)((n / 4 + 255) / 256 + 1), 256, 0, stream>>>(dq_acc.data_ptr<float>(),
                                                                              (__nv_bfloat16*)dq.data_ptr(), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dq, dk, dv};
}

}  // namespace pm

PM_DEFINE_ERROR_QUERY(pm_error_attn)
