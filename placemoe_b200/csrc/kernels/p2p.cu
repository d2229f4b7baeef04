// Peer-to-peer data-plane kernels over NVLink 5 / NVSwitch (sm_100a).
//
// Every rank owns one symmetric device buffer (mapped into every peer); a
// device table holds the peer base addresses.  Kernels store straight into
// peers' memory with 16-byte vector stores (plain st.global on the mapped
// addresses; no TMA, no multicast):
//
//   p2p_put_rows   copy rows src[src_row[i]] to peer[dst_rank[i]] + off + dst_row[i] * ld
//                  (bf16 rows; n may be a device-side count: no host synchronisation)
//   p2p_put_words  scatter 32-bit words (int32 / fp32 metadata) to peers
//   p2p_barrier    one CTA: release-store this rank's epoch into every peer's flag
//                  word, then acquire-wait until every peer's epoch reached ours.
//                  Bounded (wall-clock budget): on timeout it records kErrPeerTimeout
//                  in the sticky status block and returns; later waits then return
//                  at once and the host raises at the step's status read.
//   p2p_sum_f32    sum fp32 buffers read from several peers (replica-gradient reduction)
//   p2p_pull       bulk copy from one peer's buffer (expert-state migration)
//
// Ordering: puts of a phase are issued by kernels that complete before the
// barrier kernel on the same stream; the barrier's system-scope release
// fence + store, paired with the waiter's acquire load, makes them visible.
//
// Reference parity: replaces the NCCL all_to_all_single / batch_isend_irecv
// data plane of veomni/distributed/moe/hiermoe/all_to_all.py:725-793 and
// veomni/distributed/moe/hiermoe/expert_swap.py:6931-7107.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "peer.cuh"

namespace pm {

constexpr int kMaxPeers = 64;

// rows: warp per item, H multiple of 8 (16-byte vectors)
__global__ void __launch_bounds__(256) p2p_put_rows_kernel(const __nv_bfloat16* __restrict__ src, int H,
                                                           const int* __restrict__ src_row,
                                                           const int* __restrict__ dst_rank,
                                                           const int* __restrict__ dst_row, const int* __restrict__ n_dev,
                                                           int n_host, const long long* __restrict__ peers,
                                                           long long region_off, long long ld, int world) {
  const int n = n_dev ? min(*n_dev, n_host) : n_host;
  const int vec = H / 8;
  for (int i = blockIdx.x * 8 + (threadIdx.x >> 5); i < n; i += gridDim.x * 8) {
    const int r = dst_rank[i];
    const int dr = dst_row[i];
    const int sr = src_row ? src_row[i] : i;
    if (r < 0 || r >= world || dr < 0 || sr < 0) continue;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(peers[r] + region_off) + (size_t)dr * ld;
    const uint4* s4 = reinterpret_cast<const uint4*>(src + (size_t)sr * H);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    for (int v = threadIdx.x & 31; v < vec; v += 32) d4[v] = s4[v];
  }
}

__global__ void __launch_bounds__(256) p2p_put_words_kernel(const unsigned* __restrict__ vals,
                                                            const int* __restrict__ dst_rank,
                                                            const int* __restrict__ dst_idx,
                                                            const int* __restrict__ n_dev, int n_host,
                                                            const long long* __restrict__ peers, long long region_off,
                                                            int world) {
  const int n = n_dev ? min(*n_dev, n_host) : n_host;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int r = dst_rank[i];
    const int di = dst_idx[i];
    if (r < 0 || r >= world || di < 0) continue;
    reinterpret_cast<unsigned*>(peers[r] + region_off)[di] = vals[i];
  }
}

// Broadcast this rank's `count` words to the same offset of every peer (all-gather of a row).
__global__ void p2p_allgather_words_kernel(const unsigned* __restrict__ vals, int count,
                                           const long long* __restrict__ peers, long long region_off, int my_rank,
                                           int world) {
  for (int i = threadIdx.x; i < count * world; i += blockDim.x) {
    const int r = i / count, j = i % count;
    reinterpret_cast<unsigned*>(peers[r] + region_off)[my_rank * count + j] = vals[j];
  }
}

__global__ void p2p_barrier_kernel(const long long* __restrict__ peers, long long flags_off, int my_rank, int world,
                                   unsigned epoch, long long budget_ns, int* __restrict__ st) {
  peer_barrier_threads(peers, flags_off, my_rank, world, epoch, budget_ns, st, kWaitBarrier);
  __syncthreads();
}

// out[i] = sum over k of peer[src_rank[k]] rows (same row index i) -- used for replica-gradient
// reduction: rows = contiguous fp32 chunks.
__global__ void __launch_bounds__(256) p2p_reduce_f32_kernel(float* __restrict__ out, long long n,
                                                             const long long* __restrict__ peers,
                                                             const int* __restrict__ ranks, int nranks,
                                                             long long region_off) {
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < nranks; ++k) {
      const float4 v = reinterpret_cast<const float4*>(peers[ranks[k]] + region_off)[i];
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    reinterpret_cast<float4*>(out)[i] = acc;
  }
  if (blockIdx.x == 0)
    for (long long i = n4 * 4 + threadIdx.x; i < n; i += blockDim.x) {
      float acc = 0.f;
      for (int k = 0; k < nranks; ++k) acc += reinterpret_cast<const float*>(peers[ranks[k]] + region_off)[i];
      out[i] = acc;
    }
}

// out[i] = sum over sources j of fp32 element i at peer[src_rank[j]] + src_off[j] (byte offsets):
// the replica-gradient reduction, every copy of an expert read straight from its GPU.
__global__ void __launch_bounds__(256) p2p_sum_f32_kernel(float* __restrict__ out, long long n,
                                                          const long long* __restrict__ peers,
                                                          const int* __restrict__ src_rank,
                                                          const long long* __restrict__ src_off, int nsrc) {
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < nsrc; ++k) {
      const float4 v = reinterpret_cast<const float4*>(peers[src_rank[k]] + src_off[k])[i];
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    reinterpret_cast<float4*>(out)[i] = acc;
  }
  if (blockIdx.x == 0)
    for (long long i = n4 * 4 + threadIdx.x; i < n; i += blockDim.x) {
      float acc = 0.f;
      for (int k = 0; k < nsrc; ++k) acc += reinterpret_cast<const float*>(peers[src_rank[k]] + src_off[k])[i];
      out[i] = acc;
    }
}

// dst (local) <- peer[src_rank] + region_off, n bytes (16-byte multiple): pull copy over NVLink
__global__ void __launch_bounds__(256) p2p_pull_kernel(uint4* __restrict__ dst, const long long* __restrict__ peers,
                                                       int src_rank, long long region_off, long long n16) {
  const uint4* src = reinterpret_cast<const uint4*>(peers[src_rank] + region_off);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n16; i += (long long)gridDim.x * blockDim.x)
    dst[i] = src[i];
}

static int sm_cnt() {
  int dev, n;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

void p2p_put_rows(torch::Tensor src, c10::optional<torch::Tensor> src_row, torch::Tensor dst_rank, torch::Tensor dst_row,
                  c10::optional<torch::Tensor> n_dev, int64_t n_host, torch::Tensor peers, int64_t region_off,
                  int64_t ld) {
  PM_CHECK_CUDA(src); PM_CHECK_CUDA(dst_rank); PM_CHECK_CUDA(dst_row); PM_CHECK_CUDA(peers);
  PM_CHECK_CUDA_OPT(src_row); PM_CHECK_CUDA_OPT(n_dev);
  TORCH_CHECK(src.scalar_type() == torch::kBFloat16 && src.is_contiguous() && src.size(-1) % 8 == 0, "src bf16 rows");
  TORCH_CHECK(peers.scalar_type() == torch::kInt64 && peers.numel() <= kMaxPeers, "peer table");
  TORCH_CHECK(region_off % 16 == 0 && (ld * 2) % 16 == 0, "16-byte aligned destination rows");
  if (n_host <= 0) return;
  c10::cuda::CUDAGuard guard(src.device());
  const int grid = std::max(1, std::min((int)((n_host + 7) / 8), sm_cnt() * 4));
  p2p_put_rows_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)src.data_ptr(), (int)src.size(-1), src_row ? src_row->data_ptr<int>() : nullptr,
      dst_rank.data_ptr<int>(), dst_row.data_ptr<int>(), n_dev ? n_dev->data_ptr<int>() : nullptr, (int)n_host,
      reinterpret_cast<const long long*>(peers.data_ptr<int64_t>()), region_off,
      ld, (int)peers.numel());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void p2p_put_words(torch::Tensor vals, torch::Tensor dst_rank, torch::Tensor dst_idx, c10::optional<torch::Tensor> n_dev,
                   int64_t n_host, torch::Tensor peers, int64_t region_off) {
  PM_CHECK_CUDA(vals); PM_CHECK_CUDA(dst_rank); PM_CHECK_CUDA(dst_idx); PM_CHECK_CUDA(peers); PM_CHECK_CUDA_OPT(n_dev);
  TORCH_CHECK(vals.element_size() == 4 && vals.is_contiguous(), "32-bit words");
  if (n_host <= 0) return;
  c10::cuda::CUDAGuard guard(vals.device());
  const int grid = std::max(1, std::min((int)((n_host + 255) / 256), sm_cnt() * 4));
  p2p_put_words_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const unsigned*>(vals.data_ptr()), dst_rank.data_ptr<int>(), dst_idx.data_ptr<int>(),
      n_dev ? n_dev->data_ptr<int>() : nullptr, (int)n_host, reinterpret_cast<const long long*>(peers.data_ptr<int64_t>()),
      region_off, (int)peers.numel());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void p2p_allgather_words(torch::Tensor vals, torch::Tensor peers, int64_t region_off, int64_t my_rank) {
  PM_CHECK_CUDA(vals); PM_CHECK_CUDA(peers);
  TORCH_CHECK(vals.element_size() == 4 && vals.is_contiguous(), "32-bit words");
  c10::cuda::CUDAGuard guard(vals.device());
  p2p_allgather_words_kernel<<<1, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const unsigned*>(vals.data_ptr()), (int)vals.numel(),
      reinterpret_cast<const long long*>(peers.data_ptr<int64_t>()), region_off, (int)my_rank, (int)peers.numel());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void p2p_barrier(torch::Tensor peers, int64_t flags_off, int64_t my_rank, int64_t epoch, double timeout_s,
                 torch::Tensor status) {
  PM_CHECK_CUDA(peers); PM_CHECK_CUDA(status);
  TORCH_CHECK(peers.numel() <= kMaxPeers && my_rank < peers.numel(), "peer table");
  TORCH_CHECK(status.scalar_type() == torch::kInt32 && status.numel() >= 4, "status: int32[4]");
  c10::cuda::CUDAGuard guard(peers.device());
  p2p_barrier_kernel<<<1, 64, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const long long*>(peers.data_ptr<int64_t>()), flags_off, (int)my_rank, (int)peers.numel(),
      (unsigned)epoch, (long long)(timeout_s * 1e9), status.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void p2p_reduce_f32(torch::Tensor out, torch::Tensor peers, torch::Tensor ranks, int64_t region_off) {
  PM_CHECK_CUDA(out); PM_CHECK_CUDA(peers); PM_CHECK_CUDA(ranks);
  TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.is_contiguous(), "out fp32");
  TORCH_CHECK(ranks.scalar_type() == torch::kInt32 && region_off % 16 == 0, "ranks int32, aligned region");
  c10::cuda::CUDAGuard guard(out.device());
  const long long n = out.numel();
  const int grid = std::max(1, std::min((int)((n / 4 + 255) / 256), sm_cnt() * 4));
  p2p_reduce_f32_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      out.data_ptr<float>(), n, reinterpret_cast<const long long*>(peers.data_ptr<int64_t>()), ranks.data_ptr<int>(),
      (int)ranks.numel(), region_off);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void p2p_sum_f32(torch::Tensor out, torch::Tensor peers, torch::Tensor src_rank, torch::Tensor src_off) {
  PM_CHECK_CUDA(out); PM_CHECK_CUDA(peers); PM_CHECK_CUDA(src_rank); PM_CHECK_CUDA(src_off);
  TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.is_contiguous(), "out fp32 contiguous");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0, "out 16-byte aligned");
  TORCH_CHECK(src_rank.scalar_type() == torch::kInt32 && src_off.scalar_type() == torch::kInt64 &&
              src_rank.numel() == src_off.numel(), "src_rank int32 / src_off int64 of equal length");
  if (out.numel() == 0 || src_rank.numel() == 0) return;
  c10::cuda::CUDAGuard guard(out.device());
  const long long n = out.numel();
  const int grid = std::max(1, std::min((int)((n / 4 + 255) / 256), sm_cnt() * 4));
  p2p_sum_f32_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      out.data_ptr<float>(), n, reinterpret_cast<const long long*>(peers.data_ptr<int64_t>()),
      src_rank.data_ptr<int>(), reinterpret_cast<const long long*>(src_off.data_ptr<int64_t>()), (int)src_rank.numel());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void p2p_pull(torch::Tensor dst, torch::Tensor peers, int64_t src_rank, int64_t region_off) {
  PM_CHECK_CUDA(dst); PM_CHECK_CUDA(peers);
  TORCH_CHECK(dst.is_contiguous() && (dst.numel() * dst.element_size()) % 16 == 0 && region_off % 16 == 0,
              "16-byte multiple copy");
  c10::cuda::CUDAGuard guard(dst.device());
  const long long n16 = dst.numel() * dst.element_size() / 16;
  const int grid = std::max(1, std::min((int)((n16 + 255) / 256), sm_cnt() * 4));
  p2p_pull_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<uint4*>(dst.data_ptr()), reinterpret_cast<const long long*>(peers.data_ptr<int64_t>()),
      (int)src_rank, region_off, n16);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace pm

PM_DEFINE_ERROR_QUERY(pm_error_p2p)
