// Ulysses sequence-parallel exchange over NVLink peer memory (sm_100a).
//
// P ranks hold contiguous chunks of every sequence: rank r has tokens
// [r*Sl, (r+1)*Sl) of each of B sequences (S = P*Sl).  Attention needs whole
// sequences, so around it the activations are re-split by heads:
//
//   seq -> heads   in  [B*Sl, C] (C = heads*D on this rank's tokens)
//                  out [B*S, C/P] (every token, this rank's head group)
//   heads -> seq   the inverse.
//
// One cooperative kernel per exchange: every warp stores 16-byte vectors of
// its (token, destination) chunk of C/P elements straight into the
// destination rank's region of a symmetric buffer, a bounded grid barrier
// plus peer barrier (peer.cuh) publishes them, and every rank copies its
// region into the output tensor.  Two regions alternate between successive
// exchanges, so a rank still copying out exchange n never sees the stores of
// exchange n+1 (a peer can only start n+2 after this rank reached n+1's
// barrier).
//
// Reference parity: the all-to-all of Ulysses sequence parallelism,
// veomni/distributed/sequence_parallel/ulysses.py:64-320 (gather_seq_scatter_heads /
// gather_heads_scatter_seq), here as peer stores instead of NCCL all_to_all.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "peer.cuh"

namespace pm {

constexpr int kSpThreads = 512;
constexpr int kSpWarps = kSpThreads / 32;

struct SpArgs {
  const long long* peers;
  int P, rank, B, Sl, C;  // C = elements per token on the sequence side
  int to_heads;           // 1: seq -> heads, 0: heads -> seq
  long long off_flags, off_region;
  unsigned epoch;
  long long budget_ns;
  int* st;
  unsigned* gbar;
};

__global__ void __launch_bounds__(kSpThreads, 2)
    sp_exchange_kernel(SpArgs a, const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out) {
  __shared__ long long s_peers[64];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < a.P; i += kSpThreads) s_peers[i] = a.peers[i];
  __syncthreads();
  const int S = a.P * a.Sl, Cp = a.C / a.P;
  const int n16 = Cp / 8;  // 16-byte vectors per chunk
  const int gw = blockIdx.x * kSpWarps + warp, nw = gridDim.x * kSpWarps;
  if (a.to_heads) {
    // chunk (local token t, destination j): columns [j*Cp, (j+1)*Cp) of row t -> row b*S + rank*Sl + i of j
    const int rows = a.B * a.Sl;
    for (int c = gw; c < rows * a.P; c += nw) {
      const int t = c / a.P, j = c % a.P;
      const int b = t / a.Sl, i = t % a.Sl;
      const uint4* src = reinterpret_cast<const uint4*>(in + (size_t)t * a.C + (size_t)j * Cp);
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<char*>(s_peers[j]) + a.off_region +
                                            ((size_t)b * S + (size_t)a.rank * a.Sl + i) * Cp * 2);
      for (int v = lane; v < n16; v += 32) dst[v] = __ldcg(src + v);
    }
  } else {
    // chunk (row q of the full sequence, this rank's heads) -> rank j = pos / Sl, row b*Sl + pos % Sl,
    // columns [rank*Cp, (rank+1)*Cp)
    const int rows = a.B * S;
    for (int q = gw; q < rows; q += nw) {
      const int b = q / S, pos = q % S;
      const int j = pos / a.Sl, i = pos % a.Sl;
      const uint4* src = reinterpret_cast<const uint4*>(in + (size_t)q * Cp);
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<char*>(s_peers[j]) + a.off_region +
                                            (((size_t)b * a.Sl + i) * a.C + (size_t)a.rank * Cp) * 2);
      for (int v = lane; v < n16; v += 32) dst[v] = __ldcg(src + v);
    }
  }
  __threadfence_system();
  grid_barrier(a.gbar, 2 * a.budget_ns, a.st);
  if (blockIdx.x == 0) {
    peer_barrier_threads(s_peers, a.off_flags, a.rank, a.P, a.epoch, a.budget_ns, a.st, kWaitSpExchange);
    __syncthreads();
  }
  grid_barrier(a.gbar, 2 * a.budget_ns, a.st);
  // copy this rank's region out (same element count both ways: B*S*Cp == B*Sl*C)
  const size_t total16 = (size_t)a.B * a.Sl * a.C / 8;
  const uint4* reg = reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(s_peers[a.rank]) + a.off_region);
  uint4* o = reinterpret_cast<uint4*>(out);
  for (size_t v = (size_t)blockIdx.x * kSpThreads + tid; v < total16; v += (size_t)gridDim.x * kSpThreads)
    o[v] = __ldcg(reg + v);
}

// geo: P, rank, B, Sl, C, to_heads, off_flags, off_region
void sp_exchange(torch::Tensor in, torch::Tensor out, torch::Tensor peers, std::vector<int64_t> geo,
                 torch::Tensor scratch, torch::Tensor status, int64_t epoch, double timeout_s) {
  PM_CHECK_CUDA(in); PM_CHECK_CUDA(out); PM_CHECK_CUDA(peers); PM_CHECK_CUDA(scratch); PM_CHECK_CUDA(status);
  TORCH_CHECK(geo.size() == 8, "sp geometry: 8 values");
  SpArgs a;
  a.P = (int)geo[0]; a.rank = (int)geo[1]; a.B = (int)geo[2]; a.Sl = (int)geo[3]; a.C = (int)geo[4];
  a.to_heads = (int)geo[5]; a.off_flags = geo[6]; a.off_region = geo[7];
  TORCH_CHECK(a.P >= 1 && a.P <= 64 && peers.numel() == a.P && a.rank < a.P, "peer table");
  TORCH_CHECK(a.C % a.P == 0 && (a.C / a.P) % 8 == 0, "C / P must be a multiple of 8 elements");
  TORCH_CHECK(a.off_region % 16 == 0 && a.off_flags % 16 == 0, "16-byte aligned regions");
  TORCH_CHECK(in.scalar_type() == torch::kBFloat16 && out.scalar_type() == torch::kBFloat16 && in.is_contiguous() &&
              out.is_contiguous(), "bf16 contiguous");
  const int64_t n = (int64_t)a.B * a.Sl * a.C;
  TORCH_CHECK(in.numel() == n && out.numel() == n, "in / out hold B * Sl * C elements");
  TORCH_CHECK(status.scalar_type() == torch::kInt32 && status.numel() >= 4 && scratch.numel() >= 2, "status");
  a.peers = reinterpret_cast<const long long*>(peers.data_ptr<int64_t>());
  a.epoch = (unsigned)epoch;
  a.budget_ns = (long long)(timeout_s * 1e9);
  a.st = status.data_ptr<int>();
  a.gbar = reinterpret_cast<unsigned*>(scratch.data_ptr<int>());
  c10::cuda::CUDAGuard guard(in.device());
  int dev, sms;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const __nv_bfloat16* ip = (const __nv_bfloat16*)in.data_ptr();
  __nv_bfloat16* op = (__nv_bfloat16*)out.data_ptr();
  void* args[] = {&a, &ip, &op};
  C10_CUDA_CHECK(cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(&sp_exchange_kernel), dim3(sms),
                                             dim3(kSpThreads), args, 0, at::cuda::getCurrentCUDAStream()));
}

}  // namespace pm
