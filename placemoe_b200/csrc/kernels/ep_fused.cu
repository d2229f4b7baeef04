// Fused expert-parallel dispatch / combine over NVLink peer memory (sm_100a).
//
// One persistent, cooperatively launched kernel per phase (every CTA resident,
// one per SM); its steps are separated by bounded grid barriers, and the
// cross-GPU steps by bounded peer barriers (peer.cuh).  Rows move with 16-byte
// st.global / ld.global on peer-mapped addresses: no TMA, no multicast.
//
// Symmetric arena of one EP group (identical layout on every rank, mapped
// into every peer; byte offsets come from the host):
//   flags              barrier epochs (one word per source rank)
//   counts[2][W][B]    per-source bucket counts, B = W * S buckets (d, s)
//   layer slabs        x[cap][H] bf16 expert-contiguous inputs, meta[cap] int4,
//                      tab[cap][kpad] int32 -- one slab per MoE layer, kept
//                      until the layer's backward (the fc1 weight gradient
//                      reads x)
//   back[T][W][H] bf16 partial sums returned to the source, per (token, GPU)
//   dw[T*K] fp32       routing-weight gradients returned to the source
//   dy[cap][H] bf16    output gradients scattered in the backward
//
// ep_dispatch (forward, rank r, T tokens, top-K):
//   A  per-CTA bucket histogram of the (token, k) assignments: logical expert
//      -> (GPU d, local slot s) through this rank's mapping M[r];
//   B  CTA 0 sums the histograms and stores this rank's count row into every
//      peer; peer barrier;
//   C  from the full count matrix every rank knows each destination's
//      128/256-row aligned expert segments and where its own assignments land
//      (segment start + rows of lower ranks + stable (token, k) order).  Each
//      token's row is stored ONCE per destination GPU (dedup), at the
//      position of its first assignment there; every assignment stores a
//      16-byte record {primary position, routing weight, source rank, t*K+k};
//      the primary also stores the list of the token's positions there.  The
//      receiver zeroes its own padding rows.  Peer barrier;
//   D  the receiver copies primary rows into the positions of the token's
//      other assignments on this GPU (local HBM copies, no second NVLink
//      transfer) and extracts the routing weights.  The grouped GEMMs read
//      the slab directly: no receiver-side gather.
// ep_combine (forward combine, and the backward of the dispatch):
//   A  the expert side pre-reduces, in fp32, the rows of every (token, GPU)
//      primary and stores the bf16 partial into back[t][r] of the source
//      (plus, backward, each assignment's routing-weight gradient into dw);
//      peer barrier;
//   B  the source sums its partials per token (<= one per destination GPU).
// ep_scatter (backward of the combine): dy rows once per (token, GPU) into the
//   destinations' dy buffer, padding rows zeroed, peer barrier, local copies
//   for the other assignments.
//
// Reference parity: rank_dedup_dispatch / rank_dedup_combine,
// veomni/distributed/moe/hiermoe/all_to_all.py:2029-2263 and :2539-2564 (one
// level: a token is sent once per destination GPU and pre-reduced there).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "peer.cuh"

namespace pm {

constexpr int kEpThreads = 512;
constexpr int kEpWarps = kEpThreads / 32;
constexpr int kEpMaxBuckets = 1024;  // W * S
constexpr int kEpMaxK = 16;
constexpr int kEpMaxPeers = 64;

struct EpGeo {
  const long long* peers;  // [W] base addresses of the arena on every rank
  int W, rank, S, K, H, T, cap, align, kpad, parity;
  int E, t_cap;       // logical experts (dispatch tables), tokens the return buffers hold
  long long off_flags, off_counts, off_x, off_meta, off_tab, off_back, off_dw, off_dy;
  long long off_prim;  // layer slab: [0] count, [1..] positions of this GPU's primary rows
  unsigned epoch;     // first barrier epoch used by this launch
  long long budget_ns;
  int* st;            // sticky status block
  unsigned* gbar;     // grid barrier words [2]
  int* blk;           // [gridDim.x][B] per-CTA bucket counts (dispatch)
  unsigned long long* marks;  // optional phase timestamps (CTA 0, %globaltimer ns), nullptr = off
};

// Phase timestamp of CTA 0 (diagnostics: the kernel bench reads them to split a kernel's time).
// Slots: dispatch 0-7, combine 8-11, scatter 16-19.
PM_DEVICE void mark_phase(const EpGeo& g, int i) {
  if (g.marks != nullptr && blockIdx.x == 0 && threadIdx.x == 0) g.marks[i] = now_ns();
}

PM_DEVICE int lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return (int)m;
}

// Bit position of the n-th (0-based) set bit of m, -1 when m has fewer bits.
PM_DEVICE int nth_set_bit(unsigned m, int n) {
  for (int i = 0; i < n && m; ++i) m &= m - 1;
  return m ? __ffs(m) - 1 : -1;
}

PM_DEVICE int4 ldcg_i4(const void* p) { return __ldcg(reinterpret_cast<const int4*>(p)); }

// Warp-cooperative row copy of n16 16-byte words: eight loads in flight per lane (a 4 KB row of
// H = 2048 bf16 in one round), then four, then singles.
PM_DEVICE void warp_copy_row(uint4* __restrict__ dst, const uint4* __restrict__ src, int n16, int lane) {
  int v = lane;
  for (; v + 224 < n16; v += 256) {
    uint4 u[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) u[j] = __ldcg(src + v + 32 * j);
#pragma unroll
    for (int j = 0; j < 8; ++j) dst[v + 32 * j] = u[j];
  }
  for (; v + 96 < n16; v += 128) {
    uint4 u[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) u[j] = __ldcg(src + v + 32 * j);
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[v + 32 * j] = u[j];
  }
  for (; v < n16; v += 32) dst[v] = __ldcg(src + v);
}

// acc[0..7] += the eight bf16 values of u
PM_DEVICE void add_bf16x8(float (&acc)[8], const uint4& u) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    acc[2 * c] += bf16_lo(w[c]);
    acc[2 * c + 1] += bf16_hi(w[c]);
  }
}

// Sum in fp32 of chunk v (16 bytes) of up to kEpMaxK rows src[idx[i] * stride16 + v], i < cnt; the loads of
// eight rows are issued before their adds so a warp keeps several row reads in flight.
template <bool LDCG>
PM_DEVICE uint4 sum_rows_chunk(const uint4* __restrict__ src, const int* idx, int cnt, size_t stride16,
                               int v) {
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i0 = 0; i0 < 16; i0 += 8) {
    if (i0 < cnt) {
      uint4 u[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint4* a = src + (size_t)idx[i0 + j] * stride16 + v;
        u[j] = i0 + j < cnt ? (LDCG ? __ldcg(a) : __ldg(a)) : make_uint4(0u, 0u, 0u, 0u);  // bf16 zeros
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) add_bf16x8(acc, u[j]);
    }
  }
  return make_uint4(pack_bf16(acc[0], acc[1]), pack_bf16(acc[2], acc[3]), pack_bf16(acc[4], acc[5]),
                    pack_bf16(acc[6], acc[7]));
}

PM_DEVICE void warp_zero_row(uint4* __restrict__ dst, int n16, int lane) {
  for (int v = lane; v < n16; v += 32) dst[v] = make_uint4(0, 0, 0, 0);
}

// All threads of the grid: make this thread's stores visible system-wide, grid barrier,
// CTA 0 runs the peer barrier, grid barrier.  Returns false on a failed wait.
PM_DEVICE bool grid_peer_barrier(const EpGeo& g, const long long* s_peers, unsigned epoch, int where) {
  __threadfence_system();
  bool ok = grid_barrier(g.gbar, 2 * g.budget_ns, g.st);
  if (blockIdx.x == 0) {
    peer_barrier_threads(s_peers, g.off_flags, g.rank, g.W, epoch, g.budget_ns, g.st, where);
    __syncthreads();
  }
  ok = grid_barrier(g.gbar, 2 * g.budget_ns, g.st) && ok;
  return ok;
}

// For the K lanes of a warp holding one token's assignments (dst d, position p; p < 0 =
// dropped): the lane of the first assignment with the same destination that was not dropped.
PM_DEVICE int first_same_dest(int d, int p, int K) {
  int first = -1;
  for (int j = 0; j < K; ++j) {
    const int dj = __shfl_sync(0xffffffffu, d, j);
    const int pj = __shfl_sync(0xffffffffu, p, j);
    if (first < 0 && dj == d && pj >= 0) first = j;
  }
  return first;
}

// Bucket (destination GPU, local slot) of assignment a, or -1 when a checked index is out of range
// (the checks exist only in the bounds-checked debug build).
PM_DEVICE int bucket_of(const EpGeo& g, const int* __restrict__ idx, const int* __restrict__ dest_tab,
                        const int* __restrict__ slot_tab, int a, int* dest) {
  const int e = idx[a];
  if (!PM_PEER_INDEX_OK(g.st, e >= 0 && e < g.E)) return -1;
  const int d = dest_tab[e], s = slot_tab[e];
  if (!PM_PEER_INDEX_OK(g.st, d >= 0 && d < g.W && s >= 0 && s < g.S)) return -1;
  *dest = d;
  return d * g.S + s;
}

// ----------------------------------------------------------------------------------- dispatch
__global__ void __launch_bounds__(kEpThreads, 2)
    ep_dispatch_kernel(EpGeo g, const __nv_bfloat16* __restrict__ x, const int* __restrict__ idx,
                       const float* __restrict__ w, const int* __restrict__ dest_tab,
                       const int* __restrict__ slot_tab, int* __restrict__ pos_out, int* __restrict__ dst_out,
                       int* __restrict__ offsets_out, float* __restrict__ row_scale) {
  extern __shared__ int sm[];
  const int B = g.W * g.S;
  int* wrun = sm;                       // [kEpWarps][B]
  int* base = wrun + kEpWarps * B;      // [B]: block base, then full per-bucket base
  int* tot = base + B;                  // [B]: assignments per bucket over all sources
  int* start = tot + B;                 // [B]: segment start of bucket (d, s) at d; in phase B the
                                        // [2][J][B] stripe sums (ep_dispatch_smem sizes it)
  __shared__ long long s_peers[kEpMaxPeers];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, blk = blockIdx.x;
  const int K = g.K, S = g.S, W = g.W;
  for (int i = tid; i < W; i += kEpThreads) s_peers[i] = g.peers[i];
  for (int i = tid; i < kEpWarps * B; i += kEpThreads) wrun[i] = 0;
  __syncthreads();

  mark_phase(g, 0);
  if (blk == 0 && tid == 0)  // this layer's list of primary rows is rebuilt in phase D
    *reinterpret_cast<int*>(reinterpret_cast<char*>(s_peers[g.rank]) + g.off_prim) = 0;
  const int chunk = (g.T + G - 1) / G;
  const int t_beg = min(g.T, blk * chunk), t_end = min(g.T, t_beg + chunk);
  const int sub = (chunk + kEpWarps - 1) / kEpWarps;
  const int wt0 = min(t_end, t_beg + warp * sub), wt1 = min(t_end, wt0 + sub);

  // ---- A: per-warp histograms over the warp's tokens
  for (int a = wt0 * K + lane; a < wt1 * K; a += 32) {
    int d;
    const int b = bucket_of(g, idx, dest_tab, slot_tab, a, &d);
    if (b >= 0) atomicAdd(&wrun[warp * B + b], 1);
  }
  __syncthreads();
  for (int b = tid; b < B; b += kEpThreads) {
    int run = 0;
    for (int k = 0; k < kEpWarps; ++k) {
      const int c = wrun[k * B + b];
      wrun[k * B + b] = run;  // exclusive prefix over the warps of this CTA
      run += c;
    }
    g.blk[(size_t)blk * B + b] = run;
  }
  grid_barrier(g.gbar, 2 * g.budget_ns, g.st);
  mark_phase(g, 1);

  // ---- B: count row to every peer (CTA 0); every CTA: its base within each bucket
  int* counts_local = reinterpret_cast<int*>(s_peers[g.rank] + g.off_counts) + (size_t)g.parity * W * B;
  {
    // Every CTA sums the block counts of each bucket over the CTAs before it (its base) and over all CTAs
    // (the totals, sent by CTA 0).  Threads split the blocks into J stripes per bucket, four independent
    // loads in flight each, then one thread per bucket adds the stripes: a serial walk over ~150 L2
    // reads per thread would cost ~100 us of latency.
    const int J = B >= kEpThreads ? 1 : kEpThreads / B;
    int* part_below = start;  // [J][B] (start / tot are not used before phase C) -- see the smem plan
    int* part_all = start + J * B;
    for (int i = tid; i < B * J; i += kEpThreads) {
      const int b = i % B, j = i / B;
      int below = 0, all = 0, k = j;
      for (; k + 3 * J < G; k += 4 * J) {
        const int c0 = __ldcg(&g.blk[(size_t)k * B + b]), c1 = __ldcg(&g.blk[(size_t)(k + J) * B + b]);
        const int c2 = __ldcg(&g.blk[(size_t)(k + 2 * J) * B + b]), c3 = __ldcg(&g.blk[(size_t)(k + 3 * J) * B + b]);
        all += c0 + c1 + c2 + c3;
        below += (k < blk ? c0 : 0) + (k + J < blk ? c1 : 0) + (k + 2 * J < blk ? c2 : 0) + (k + 3 * J < blk ? c3 : 0);
      }
      for (; k < G; k += J) {
        const int c = __ldcg(&g.blk[(size_t)k * B + b]);
        all += c;
        below += k < blk ? c : 0;
      }
      part_below[j * B + b] = below;
      part_all[j * B + b] = all;
    }
    __syncthreads();
    for (int b = tid; b < B; b += kEpThreads) {
      int below = 0, all = 0;
      for (int j = 0; j < J; ++j) {
        below += part_below[j * B + b];
        all += part_all[j * B + b];
      }
      base[b] = below;
      if (blk == 0)
        for (int r = 0; r < W; ++r)
          reinterpret_cast<int*>(s_peers[r] + g.off_counts)[(size_t)g.parity * W * B + (size_t)g.rank * B + b] = all;
    }
  }
  grid_peer_barrier(g, s_peers, g.epoch, kWaitEpCounts);
  mark_phase(g, 2);

  // ---- C: segment layout of every destination, positions, stores
  for (int b = tid; b < B; b += kEpThreads) {
    int t = 0, below = 0;
    for (int src = 0; src < W; ++src) {
      const int c = __ldcg(&counts_local[(size_t)src * B + b]);
      t += c;
      if (src < g.rank) below += c;
    }
    tot[b] = t;
    base[b] += below;
  }
  __syncthreads();
  for (int d = tid; d < W; d += kEpThreads) {
    int run = 0;
    for (int s = 0; s < S; ++s) {
      start[d * S + s] = run;
      run += (tot[d * S + s] + g.align - 1) / g.align * g.align;
    }
  }
  __syncthreads();
  for (int b = tid; b < B; b += kEpThreads) {
    const int full = base[b] + start[b];
    for (int k = 0; k < kEpWarps; ++k) wrun[k * B + b] += full;
  }
  // this rank's own expert segments (receiver side)
  const int* my_start = start + g.rank * S;
  const int* my_tot = tot + g.rank * S;
  const int n_rows = my_start[S - 1] + (my_tot[S - 1] + g.align - 1) / g.align * g.align;
  if (blk == 0) {
    for (int s = tid; s <= S; s += kEpThreads) offsets_out[s] = min(s < S ? my_start[s] : n_rows, g.cap);
    if (tid == 0) atomicMax(g.st + 2, n_rows);
  }
  __syncthreads();

  mark_phase(g, 3);
  // positions: stable (token, k) order within every bucket
  for (int a0 = wt0 * K; a0 < wt1 * K; a0 += 32) {
    const int a = a0 + lane;
    const bool valid = a < wt1 * K;
    int b = -1, d = 0;
    if (valid) b = bucket_of(g, idx, dest_tab, slot_tab, a, &d);
    const unsigned same = __match_any_sync(0xffffffffu, b);
    const int rnk = __popc(same & (unsigned)lanemask_lt());
    const int p = b >= 0 ? wrun[warp * B + b] + rnk : -1;
    __syncwarp();
    if (b >= 0 && rnk == 0) wrun[warp * B + b] += __popc(same);
    __syncwarp();
    if (valid) {
      pos_out[a] = p < g.cap ? p : -1;  // -1: dropped (beyond the slab) or a bad index
      dst_out[a] = d;
    }
  }
  __syncthreads();

  mark_phase(g, 4);
  const int n16 = g.H / 8;
  for (int t = t_beg + warp; t < t_end; t += kEpWarps) {
    const int a = t * K + lane;
    int d = -1, p = -1;
    float wt = 0.f;
    if (lane < K) {
      d = dst_out[a];
      p = pos_out[a];
      wt = w[a];
    }
    const int first = first_same_dest(d, p, K);
    const int prim = __shfl_sync(0xffffffffu, p, first < 0 ? 0 : first);
    const bool is_primary = lane < K && p >= 0 && first == lane;
    if (lane < K && p >= 0) {
      char* peer = reinterpret_cast<char*>(s_peers[d]);
      *reinterpret_cast<int4*>(peer + g.off_meta + (size_t)p * 16) =
          make_int4(prim, __float_as_int(wt), g.rank, a);
    }
    // positions of this token's assignments on each destination, in k order
    unsigned mine = 0;
    for (int j = 0; j < K; ++j) {
      const int dj = __shfl_sync(0xffffffffu, d, j);
      const int pj = __shfl_sync(0xffffffffu, p, j);
      if (dj == d && pj >= 0) mine |= 1u << j;
    }
    for (int c = 0; c < g.kpad; c += 4) {
      int v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int nth = c + i;
        const int src = nth_set_bit(mine, nth);
        const int pv = __shfl_sync(0xffffffffu, p, src < 0 ? 0 : src);
        v[i] = src < 0 ? -1 : pv;
      }
      if (is_primary)
        *reinterpret_cast<int4*>(reinterpret_cast<char*>(s_peers[d]) + g.off_tab + ((size_t)p * g.kpad + c) * 4) =
            make_int4(v[0], v[1], v[2], v[3]);
    }
    unsigned prims = __ballot_sync(0xffffffffu, is_primary);
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * g.H);
    while (prims) {
      const int j = __ffs(prims) - 1;
      prims &= prims - 1;
      const int dj = __shfl_sync(0xffffffffu, d, j);
      const int pj = __shfl_sync(0xffffffffu, p, j);
      uint4* dstrow = reinterpret_cast<uint4*>(reinterpret_cast<char*>(s_peers[dj]) + g.off_x + (size_t)pj * g.H * 2);
      warp_copy_row(dstrow, src, n16, lane);
    }
  }

  // receiver: padding rows of this rank's segments
  {
    char* me = reinterpret_cast<char*>(s_peers[g.rank]);
    const int gw = blk * kEpWarps + warp, nw = G * kEpWarps;
    for (int s = 0; s < S; ++s) {
      const int lo = my_start[s] + my_tot[s];
      const int hi = min(s + 1 < S ? my_start[s + 1] : n_rows, g.cap);
      for (int q = lo + gw; q < hi; q += nw) {
        warp_zero_row(reinterpret_cast<uint4*>(me + g.off_x + (size_t)q * g.H * 2), n16, lane);
        if (lane == 0) *reinterpret_cast<int4*>(me + g.off_meta + (size_t)q * 16) = make_int4(-1, 0, -1, -1);
      }
    }
  }
  mark_phase(g, 5);
  grid_peer_barrier(g, s_peers, g.epoch + 1, kWaitEpRows);
  mark_phase(g, 6);

  // ---- D: local copies for the other assignments of a token on this GPU; routing weights
  {
    char* me = reinterpret_cast<char*>(s_peers[g.rank]);
    const int n = min(n_rows, g.cap);
    for (int q = blk * kEpWarps + warp; q < n; q += G * kEpWarps) {
      const int4 m = ldcg_i4(me + g.off_meta + (size_t)q * 16);
      const bool ok = m.x < 0 || PM_PEER_INDEX_OK(g.st, m.x < n);
      if (lane == 0) {
        row_scale[q] = (m.x >= 0 && ok) ? __int_as_float(m.y) : 0.f;
        if (m.x == q) {  // a primary: the combine pre-reduces from it (list order is irrelevant to results)
          int* prim = reinterpret_cast<int*>(me + g.off_prim);
          prim[1 + atomicAdd(prim, 1)] = q;
        }
      }
      if (m.x >= 0 && m.x != q && ok)
        warp_copy_row(reinterpret_cast<uint4*>(me + g.off_x + (size_t)q * g.H * 2),
                      reinterpret_cast<const uint4*>(me + g.off_x + (size_t)m.x * g.H * 2), n16, lane);
    }
  }
  mark_phase(g, 7);
}

// ------------------------------------------------------------------------------------ combine
__global__ void __launch_bounds__(kEpThreads, 2)
    ep_combine_kernel(EpGeo g, const __nv_bfloat16* __restrict__ rows, const float* __restrict__ dscale,
                      const int* __restrict__ pos, const int* __restrict__ dst, const int* __restrict__ offsets,
                      __nv_bfloat16* __restrict__ out, float* __restrict__ dw_out) {
  __shared__ long long s_peers[kEpMaxPeers];
  __shared__ int s_list[kEpWarps][kEpMaxK];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, blk = blockIdx.x;
  const int K = g.K, W = g.W, n16 = g.H / 8;
  for (int i = tid; i < W; i += kEpThreads) s_peers[i] = g.peers[i];
  __syncthreads();
  char* me = reinterpret_cast<char*>(s_peers[g.rank]);
  const int n = min(offsets[g.S], g.cap);
  mark_phase(g, 8);

  // ---- A: pre-reduce every primary's rows, partial sum back to the source.  Warps walk the list of
  // primaries the dispatch built (even work per warp: a primary's rows sit in different expert segments,
  // so walking positions would give some warps many primaries and others none).
  const int* prim = reinterpret_cast<const int*>(me + g.off_prim);
  const int nprim = min(__ldcg(prim), n);
  for (int i = blk * kEpWarps + warp; i < nprim; i += G * kEpWarps) {
    const int q = __ldcg(prim + 1 + i);
    if (!PM_PEER_INDEX_OK(g.st, q >= 0 && q < n)) continue;
    const int4 m = ldcg_i4(me + g.off_meta + (size_t)q * 16);
    if (m.x != q) continue;
    if (!PM_PEER_INDEX_OK(g.st, m.z >= 0 && m.z < W && m.w >= 0 && m.w < g.t_cap * K)) continue;
    const int* tab = reinterpret_cast<const int*>(me + g.off_tab) + (size_t)q * g.kpad;
    int* list = s_list[warp];  // this primary's rows (shared memory keeps them out of registers)
    int cnt = 0;
    __syncwarp();  // every lane is done with the previous primary's list
#pragma unroll
    for (int j = 0; j < kEpMaxK; ++j) {
      int v = j < g.kpad ? __ldcg(tab + j) : -1;
      if (v >= 0 && !PM_PEER_INDEX_OK(g.st, v < n)) v = -1;
      cnt += (v >= 0 && cnt == j) ? 1 : 0;
      if (lane == 0) list[j] = v >= 0 ? v : 0;
    }
    __syncwarp();
    if (dscale != nullptr && lane < cnt) {  // routing-weight gradient of every assignment of the token here
      const int qi = list[lane];
      const int4 mi = ldcg_i4(me + g.off_meta + (size_t)qi * 16);
      if (PM_PEER_INDEX_OK(g.st, mi.w >= 0 && mi.w < g.t_cap * K))
        reinterpret_cast<float*>(s_peers[m.z] + g.off_dw)[mi.w] = dscale[qi];
    }
    const int t = m.w / K;
    uint4* dstrow = reinterpret_cast<uint4*>(reinterpret_cast<char*>(s_peers[m.z]) + g.off_back +
                                             ((size_t)t * W + g.rank) * g.H * 2);
    const uint4* src = reinterpret_cast<const uint4*>(rows);
    if (cnt == 1)  // one assignment of the token on this GPU: the partial is its row
      warp_copy_row(dstrow, src + (size_t)list[0] * n16, n16, lane);
    else
      for (int v = lane; v < n16; v += 32) dstrow[v] = sum_rows_chunk<false>(src, list, cnt, n16, v);
  }
  mark_phase(g, 9);
  grid_peer_barrier(g, s_peers, g.epoch, kWaitEpCombine);
  mark_phase(g, 10);

  // ---- B: per token, the sum of its partials (one per destination GPU)
  for (int t = blk * kEpWarps + warp; t < g.T; t += G * kEpWarps) {
    int d = -1, p = -1;
    if (lane < K) {
      d = dst[t * K + lane];
      p = pos[t * K + lane];
      if (p >= 0 && !PM_PEER_INDEX_OK(g.st, d >= 0 && d < W)) p = -1;
    }
    const unsigned dmask = __reduce_or_sync(0xffffffffu, (lane < K && p >= 0) ? (1u << d) : 0u);
    if (dw_out != nullptr && lane < K)
      dw_out[t * K + lane] = p >= 0 ? __ldcg(reinterpret_cast<const float*>(me + g.off_dw) + t * K + lane) : 0.f;
    const uint4* back = reinterpret_cast<const uint4*>(me + g.off_back + (size_t)t * W * g.H * 2);
    int* dl = s_list[warp];  // destination GPUs of this token (at most K), lowest first
    unsigned mm = dmask;
    const int nd = min(__popc(dmask), kEpMaxK);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < kEpMaxK; ++i) {
      if (lane == 0) dl[i] = mm ? __ffs(mm) - 1 : 0;
      mm &= mm - 1;
    }
    __syncwarp();
    uint4* orow = reinterpret_cast<uint4*>(out + (size_t)t * g.H);
    if (nd == 1)  // one destination GPU: the token's output is its partial
      warp_copy_row(orow, back + (size_t)dl[0] * n16, n16, lane);
    else
      for (int v = lane; v < n16; v += 32) orow[v] = sum_rows_chunk<true>(back, dl, nd, n16, v);
  }
  mark_phase(g, 11);
}

// ------------------------------------------------------------------------------------ scatter
__global__ void __launch_bounds__(kEpThreads, 2)
    ep_scatter_kernel(EpGeo g, const __nv_bfloat16* __restrict__ dy, const int* __restrict__ pos,
                      const int* __restrict__ dst, const int* __restrict__ offsets) {
  __shared__ long long s_peers[kEpMaxPeers];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, blk = blockIdx.x;
  const int K = g.K, n16 = g.H / 8;
  for (int i = tid; i < g.W; i += kEpThreads) s_peers[i] = g.peers[i];
  __syncthreads();
  char* me = reinterpret_cast<char*>(s_peers[g.rank]);
  const int n = min(offsets[g.S], g.cap);
  mark_phase(g, 16);

  // ---- A: dy once per (token, destination GPU); padding rows of this rank zeroed
  for (int t = blk * kEpWarps + warp; t < g.T; t += G * kEpWarps) {
    int d = -1, p = -1;
    if (lane < K) {
      d = dst[t * K + lane];
      p = pos[t * K + lane];
      if (p >= 0 && !PM_PEER_INDEX_OK(g.st, d >= 0 && d < g.W && p < g.cap)) p = -1;
    }
    const int first = first_same_dest(d, p, K);
    unsigned prims = __ballot_sync(0xffffffffu, lane < K && p >= 0 && first == lane);
    const uint4* src = reinterpret_cast<const uint4*>(dy + (size_t)t * g.H);
    while (prims) {
      const int j = __ffs(prims) - 1;
      prims &= prims - 1;
      const int dj = __shfl_sync(0xffffffffu, d, j);
      const int pj = __shfl_sync(0xffffffffu, p, j);
      warp_copy_row(reinterpret_cast<uint4*>(reinterpret_cast<char*>(s_peers[dj]) + g.off_dy + (size_t)pj * g.H * 2),
                    src, n16, lane);
    }
  }
  for (int q = blk * kEpWarps + warp; q < n; q += G * kEpWarps) {
    const int4 m = ldcg_i4(me + g.off_meta + (size_t)q * 16);
    if (m.x < 0) warp_zero_row(reinterpret_cast<uint4*>(me + g.off_dy + (size_t)q * g.H * 2), n16, lane);
  }
  mark_phase(g, 17);
  grid_peer_barrier(g, s_peers, g.epoch, kWaitEpScatter);
  mark_phase(g, 18);

  // ---- B: local copies for the token's other assignments on this GPU
  for (int q = blk * kEpWarps + warp; q < n; q += G * kEpWarps) {
    const int4 m = ldcg_i4(me + g.off_meta + (size_t)q * 16);
    if (m.x >= 0 && m.x != q && PM_PEER_INDEX_OK(g.st, m.x < n))
      warp_copy_row(reinterpret_cast<uint4*>(me + g.off_dy + (size_t)q * g.H * 2),
                    reinterpret_cast<const uint4*>(me + g.off_dy + (size_t)m.x * g.H * 2), n16, lane);
  }
  mark_phase(g, 19);
}

// ------------------------------------------------------------------------------------ host side
// geo (int64): W, rank, S, K, H, T_cap, cap, align, kpad, parity,
//              off_flags, off_counts, off_x, off_meta, off_tab, off_back, off_dw, off_dy, off_prim
// Phase-timestamp buffer for diagnostics (set by ep_phase_marks; nullptr = no timestamps).
static unsigned long long* g_ep_marks = nullptr;

void ep_phase_marks(c10::optional<torch::Tensor> buf) {
  if (!buf.has_value()) {
    g_ep_marks = nullptr;
    return;
  }
  PM_CHECK_CUDA(*buf);
  TORCH_CHECK(buf->scalar_type() == torch::kInt64 && buf->numel() >= 24, "marks: int64[24]");
  g_ep_marks = reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>());
}

static EpGeo make_geo(const std::vector<int64_t>& v, const torch::Tensor& peers, const torch::Tensor& scratch,
                      const torch::Tensor& status, int64_t epoch, double timeout_s, int T) {
  TORCH_CHECK(v.size() == 19, "ep geometry: 19 values");
  PM_CHECK_CUDA(peers); PM_CHECK_CUDA(scratch); PM_CHECK_CUDA(status);
  TORCH_CHECK(peers.scalar_type() == torch::kInt64 && peers.numel() == v[0] && v[0] <= kEpMaxPeers, "peer table");
  TORCH_CHECK(status.scalar_type() == torch::kInt32 && status.numel() >= 4, "status: int32[4]");
  TORCH_CHECK(scratch.scalar_type() == torch::kInt32, "scratch int32");
  EpGeo g;
  g.peers = reinterpret_cast<const long long*>(peers.data_ptr<int64_t>());
  g.W = (int)v[0]; g.rank = (int)v[1]; g.S = (int)v[2]; g.K = (int)v[3]; g.H = (int)v[4];
  g.T = T; g.cap = (int)v[6]; g.align = (int)v[7]; g.kpad = (int)v[8]; g.parity = (int)v[9];
  g.E = 0; g.t_cap = (int)v[5];
  g.off_flags = v[10]; g.off_counts = v[11]; g.off_x = v[12]; g.off_meta = v[13]; g.off_tab = v[14];
  g.off_back = v[15]; g.off_dw = v[16]; g.off_dy = v[17]; g.off_prim = v[18];
  TORCH_CHECK(T <= v[5], "more tokens than the arena holds");
  TORCH_CHECK(g.K >= 1 && g.K <= kEpMaxK && g.kpad % 4 == 0 && g.kpad >= g.K && g.kpad <= kEpMaxK, "top-k");
  TORCH_CHECK(g.W * g.S <= kEpMaxBuckets && g.W <= 32, "W * S <= 1024 buckets, W <= 32");
  TORCH_CHECK(g.H % 8 == 0 && g.align > 0 && g.cap % g.align == 0, "geometry");
  for (int i = 10; i < 19; ++i) TORCH_CHECK(v[i] % 16 == 0, "16-byte aligned arena regions");
  g.epoch = (unsigned)epoch;
  g.budget_ns = (long long)(timeout_s * 1e9);
  g.st = status.data_ptr<int>();
  g.gbar = reinterpret_cast<unsigned*>(scratch.data_ptr<int>());
  g.blk = scratch.data_ptr<int>() + 2;
  g.marks = g_ep_marks;
  return g;
}

// Dynamic shared memory of the dispatch kernel: warp counters, base and totals, then the area that
// holds the segment starts in phase C and the [2][J][B] stripe sums of phase B.
static size_t ep_dispatch_smem(int B) {
  const int J = B >= kEpThreads ? 1 : kEpThreads / B;
  return (size_t)(kEpWarps + 2) * B * sizeof(int) + (size_t)std::max(B, 2 * J * B) * sizeof(int);
}

static int ep_grid(const void* fn, size_t smem) {
  int dev, sms, per = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  C10_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, fn, kEpThreads, smem));
  TORCH_CHECK(per >= 1, "EP kernel does not fit on an SM");
  return sms;  // one CTA per SM: room stays for the side-stream kernels
}

static void launch_coop(const void* fn, int grid, size_t smem, void** args) {
  C10_CUDA_CHECK(cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(kEpThreads), args, smem,
                                             at::cuda::getCurrentCUDAStream()));
}

int64_t ep_scratch_ints(int64_t world, int64_t slots) {
  int dev, sms;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  return 2 + (int64_t)sms * world * slots;
}

void ep_dispatch(torch::Tensor x, torch::Tensor idx, torch::Tensor w, torch::Tensor dest_tab, torch::Tensor slot_tab,
                 torch::Tensor peers, std::vector<int64_t> geo, torch::Tensor scratch, torch::Tensor status,
                 int64_t epoch, double timeout_s, torch::Tensor pos, torch::Tensor dst, torch::Tensor offsets,
                 torch::Tensor row_scale) {
  PM_CHECK_CUDA(x); PM_CHECK_CUDA(idx); PM_CHECK_CUDA(w); PM_CHECK_CUDA(dest_tab); PM_CHECK_CUDA(slot_tab);
  PM_CHECK_CUDA(pos); PM_CHECK_CUDA(dst); PM_CHECK_CUDA(offsets); PM_CHECK_CUDA(row_scale);
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && x.is_contiguous() && x.dim() == 2, "x: [T, H] bf16");
  const int T = (int)x.size(0);
  EpGeo g = make_geo(geo, peers, scratch, status, epoch, timeout_s, T);
  TORCH_CHECK(x.size(1) == g.H, "hidden size");
  TORCH_CHECK(idx.scalar_type() == torch::kInt32 && idx.is_contiguous() && idx.numel() == (int64_t)T * g.K, "idx");
  TORCH_CHECK(w.scalar_type() == torch::kFloat32 && w.is_contiguous() && w.numel() == idx.numel(), "w");
  TORCH_CHECK(dest_tab.scalar_type() == torch::kInt32 && slot_tab.scalar_type() == torch::kInt32 &&
              dest_tab.numel() == slot_tab.numel(), "mapping tables");
  TORCH_CHECK(pos.numel() == idx.numel() && dst.numel() == idx.numel() && pos.scalar_type() == torch::kInt32 &&
              dst.scalar_type() == torch::kInt32, "pos / dst: int32 [T, K]");
  TORCH_CHECK(offsets.numel() == g.S + 1 && offsets.scalar_type() == torch::kInt32, "offsets: int32 [S+1]");
  TORCH_CHECK(row_scale.numel() >= g.cap && row_scale.scalar_type() == torch::kFloat32, "row_scale: fp32 [cap]");
  g.E = (int)dest_tab.numel();
  const int B = g.W * g.S;
  const size_t smem = ep_dispatch_smem(B);
  const void* fn = reinterpret_cast<const void*>(&ep_dispatch_kernel);
  C10_CUDA_CHECK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int grid = ep_grid(fn, smem);
  TORCH_CHECK(scratch.numel() >= 2 + (int64_t)grid * B, "scratch too small");
  c10::cuda::CUDAGuard guard(x.device());
  const __nv_bfloat16* xp = (const __nv_bfloat16*)x.data_ptr();
  const int* ip = idx.data_ptr<int>();
  const float* wp = w.data_ptr<float>();
  const int* dp = dest_tab.data_ptr<int>();
  const int* sp = slot_tab.data_ptr<int>();
  int* pp = pos.data_ptr<int>();
  int* dsp = dst.data_ptr<int>();
  int* op = offsets.data_ptr<int>();
  float* rp = row_scale.data_ptr<float>();
  void* args[] = {&g, &xp, &ip, &wp, &dp, &sp, &pp, &dsp, &op, &rp};
  launch_coop(fn, grid, smem, args);
}

void ep_combine(torch::Tensor rows, c10::optional<torch::Tensor> dscale, torch::Tensor pos, torch::Tensor dst,
                torch::Tensor offsets, torch::Tensor peers, std::vector<int64_t> geo, torch::Tensor scratch,
                torch::Tensor status, int64_t epoch, double timeout_s, torch::Tensor out,
                c10::optional<torch::Tensor> dw_out) {
  PM_CHECK_CUDA(rows); PM_CHECK_CUDA(pos); PM_CHECK_CUDA(dst); PM_CHECK_CUDA(offsets); PM_CHECK_CUDA(out);
  PM_CHECK_CUDA_OPT(dscale); PM_CHECK_CUDA_OPT(dw_out);
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.is_contiguous() && out.dim() == 2, "out: [T, H] bf16");
  const int T = (int)out.size(0);
  EpGeo g = make_geo(geo, peers, scratch, status, epoch, timeout_s, T);
  TORCH_CHECK(rows.scalar_type() == torch::kBFloat16 && rows.is_contiguous() && rows.size(0) >= g.cap &&
              rows.size(1) == g.H, "rows: [cap, H] bf16");
  TORCH_CHECK(pos.numel() == (int64_t)T * g.K && dst.numel() == pos.numel(), "pos / dst");
  TORCH_CHECK(dscale.has_value() == dw_out.has_value(), "dscale and dw_out go together");
  if (dscale.has_value()) {
    TORCH_CHECK(dscale->scalar_type() == torch::kFloat32 && dscale->numel() >= g.cap, "dscale fp32 [cap]");
    TORCH_CHECK(dw_out->scalar_type() == torch::kFloat32 && dw_out->numel() == pos.numel(), "dw_out fp32 [T, K]");
  }
  const void* fn = reinterpret_cast<const void*>(&ep_combine_kernel);
  const int grid = ep_grid(fn, 0);
  c10::cuda::CUDAGuard guard(out.device());
  const __nv_bfloat16* rp = (const __nv_bfloat16*)rows.data_ptr();
  const float* dsp = dscale.has_value() ? dscale->data_ptr<float>() : nullptr;
  const int* pp = pos.data_ptr<int>();
  const int* dp = dst.data_ptr<int>();
  const int* op = offsets.data_ptr<int>();
  __nv_bfloat16* outp = (__nv_bfloat16*)out.data_ptr();
  float* dwp = dw_out.has_value() ? dw_out->data_ptr<float>() : nullptr;
  void* args[] = {&g, &rp, &dsp, &pp, &dp, &op, &outp, &dwp};
  launch_coop(fn, grid, 0, args);
}

void ep_scatter(torch::Tensor dy, torch::Tensor pos, torch::Tensor dst, torch::Tensor offsets, torch::Tensor peers,
                std::vector<int64_t> geo, torch::Tensor scratch, torch::Tensor status, int64_t epoch,
                double timeout_s) {
  PM_CHECK_CUDA(dy); PM_CHECK_CUDA(pos); PM_CHECK_CUDA(dst); PM_CHECK_CUDA(offsets);
  TORCH_CHECK(dy.scalar_type() == torch::kBFloat16 && dy.is_contiguous() && dy.dim() == 2, "dy: [T, H] bf16");
  const int T = (int)dy.size(0);
  EpGeo g = make_geo(geo, peers, scratch, status, epoch, timeout_s, T);
  TORCH_CHECK(dy.size(1) == g.H && pos.numel() == (int64_t)T * g.K && dst.numel() == pos.numel(), "shapes");
  const void* fn = reinterpret_cast<const void*>(&ep_scatter_kernel);
  const int grid = ep_grid(fn, 0);
  c10::cuda::CUDAGuard guard(dy.device());
  const __nv_bfloat16* dyp = (const __nv_bfloat16*)dy.data_ptr();
  const int* pp = pos.data_ptr<int>();
  const int* dp = dst.data_ptr<int>();
  const int* op = offsets.data_ptr<int>();
  void* args[] = {&g, &dyp, &pp, &dp, &op};
  launch_coop(fn, grid, 0, args);
}

}  // namespace pm
