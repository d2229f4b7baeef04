// tcgen05 GEMM entry points: expert-grouped forward / data-gradient GEMMs.
// The kernel template, tile scheduler and epilogues are in gemm_sm100.cuh.
#include "gemm_sm100.cuh"

namespace pm {

// Expert fc1 forward: h[rows, I] = scale[row] * silu(x W1_gate^T) * (x W1_up^T)
// x: [rows, H] dispatched tokens, expert segments at group_offsets (multiples of 128).
// w1: [E, 2I, H] (gate rows first, then up rows).  gu_out (optional): [rows, 2I].
// align: the segment alignment of `offsets` (128, or 256 to run on CTA pairs).
// gather_idx (optional, int32 [rows]): A row r is x[gather_idx[r]] (fetched by TMA row
// gathers; < 0 marks padding) instead of x[r].
void moe_fc1_swiglu(torch::Tensor x, torch::Tensor w1, torch::Tensor offsets, torch::Tensor scale, torch::Tensor h,
                    c10::optional<torch::Tensor> gu_out, int64_t align, c10::optional<torch::Tensor> gather_idx) {
  TORCH_CHECK(align == 128 || align == 256, "segment alignment must be 128 or 256");
  const bool gather = gather_idx.has_value();
  if (gather) {
    TORCH_CHECK(gather_idx->is_cuda() && gather_idx->scalar_type() == torch::kInt32 && gather_idx->is_contiguous(),
                "gather_idx must be a contiguous int32 CUDA tensor");
    TORCH_CHECK((reinterpret_cast<uintptr_t>(gather_idx->data_ptr()) & 15) == 0, "gather_idx must be 16-byte aligned");
  }
  const int64_t rows = gather ? gather_idx->numel() : x.size(0);
  check_bf16_2d(x, "x");
  TORCH_CHECK(w1.dim() == 3 && w1.is_contiguous() && w1.scalar_type() == torch::kBFloat16, "w1 must be [E,2I,H] bf16");
  const int64_t E = w1.size(0), I2 = w1.size(1), H = w1.size(2);
  const int64_t I = I2 / 2;
  TORCH_CHECK(x.size(1) == H, "x/w1 hidden mismatch");
  TORCH_CHECK(I % 128 == 0, "moe intermediate size must be a multiple of 128");
  TORCH_CHECK(E <= kMaxGroups, "too many experts");
  TORCH_CHECK(offsets.scalar_type() == torch::kInt32 && offsets.numel() == E + 1, "offsets must be int32 [E+1]");
  TORCH_CHECK(h.size(0) == rows && h.size(1) == I && h.stride(1) == 1, "h shape");
  PM_CHECK_CUDA(w1); PM_CHECK_CUDA(offsets); PM_CHECK_CUDA(scale); PM_CHECK_CUDA(h); PM_CHECK_CUDA_OPT(gu_out);
  TORCH_CHECK(scale.scalar_type() == torch::kFloat32 && scale.numel() >= rows, "scale must be fp32 [rows]");
  c10::cuda::CUDAGuard guard(x.device());
  GemmArgs args = blank_args();
  args.M = (int)rows; args.N = (int)I2; args.K = (int)H; args.num_groups = (int)E;
  if (gather) args.gather_idx = gather_idx->data_ptr<int>();
  args.group_offsets = offsets.data_ptr<int>();
  args.raster = 1;  // an expert's weights (<= tens of MB) stay in L2 while its rows stream once
  args.D = h.data_ptr(); args.ldd = h.stride(0);
  args.row_scale = scale.data_ptr<float>();
  args.inter = (int)I;
  if (gu_out.has_value()) {
    check_bf16_2d(*gu_out, "gu_out");
    args.aux_out = reinterpret_cast<__nv_bfloat16*>(gu_out->data_ptr());
    args.ld_aux_out = gu_out->stride(0);
  }
  CUtensorMap ta = make_tmap_2d_bf16(x.data_ptr(), x.size(0), H, x.stride(0), 64, gather ? 1 : 128);
  CUtensorMap tb = make_tmap_3d_bf16(w1.data_ptr(), E, I2, H, H, I2 * H, 64, 128);
  check_bf16_2d(h, "h");
  CUtensorMap th = make_tmap_bf16_epi(h.data_ptr(), h.size(0), I, h.stride(0));
  CUtensorMap tg;
  if (gu_out.has_value()) tg = make_tmap_bf16_epi(gu_out->data_ptr(), gu_out->size(0), I2, gu_out->stride(0));
  const CUtensorMap* tgp = gu_out.has_value() ? &tg : nullptr;
  if (align == 256) {
    const int grid = std::max(1, std::min((int)((rows / 256) * (I / 128)), num_pairs()));
    if (gather) launch<256, false, false, kGroupM, kSwiGLU, true, true, true>(ta, tb, args, grid, &th, tgp);
    else launch<256, false, false, kGroupM, kSwiGLU, true, true>(ta, tb, args, grid, &th, tgp);
    return;
  }
  const int grid = std::max(1, std::min((int)((rows / BM) * (I / 128)), num_sms()));
  if (gather) launch<256, false, false, kGroupM, kSwiGLU, true, false, true>(ta, tb, args, grid, &th, tgp);
  else launch<256, false, false, kGroupM, kSwiGLU, true>(ta, tb, args, grid, &th, tgp);
}

// Expert GEMM with per-expert B, grouped over rows of A.
//   b_mn = false: out[rows, N] = a[rows, K] . w[e]^T, w: [E, N, K]  (fc2 forward)
//   b_mn = true : out[rows, N] = a[rows, K] . w[e],   w: [E, K, N]  (data gradients)
void moe_grouped_gemm(torch::Tensor a, torch::Tensor w, torch::Tensor offsets, torch::Tensor out, bool b_mn,
                      int64_t align) {
  TORCH_CHECK(align == 128 || align == 256, "segment alignment must be 128 or 256");
  const bool pair = align == 256;
  check_bf16_2d(a, "a");
  check_bf16_2d(out, "out");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16, "out must be bf16");
  TORCH_CHECK(w.dim() == 3 && w.is_contiguous() && w.scalar_type() == torch::kBFloat16, "w must be 3-D bf16");
  const int64_t E = w.size(0);
  const int64_t N = b_mn ? w.size(2) : w.size(1);
  const int64_t K = b_mn ? w.size(1) : w.size(2);
  TORCH_CHECK(a.size(1) == K && out.size(1) == N && out.size(0) == a.size(0), "shape mismatch");
  TORCH_CHECK(N % 8 == 0, "N must be a multiple of 8");
  TORCH_CHECK(E <= kMaxGroups && offsets.numel() == E + 1 && offsets.scalar_type() == torch::kInt32, "offsets");
  PM_CHECK_CUDA(w); PM_CHECK_CUDA(offsets);
  c10::cuda::CUDAGuard guard(a.device());
  GemmArgs args = blank_args();
  args.M = (int)a.size(0); args.N = (int)N; args.K = (int)K; args.num_groups = (int)E;
  args.group_offsets = offsets.data_ptr<int>();
  args.raster = 1;  // an expert's weights (<= tens of MB) stay in L2 while its rows stream once
  args.D = out.data_ptr(); args.ldd = out.stride(0);
  CUtensorMap ta = make_tmap_2d_bf16(a.data_ptr(), a.size(0), K, a.stride(0), 64, 128);
  CUtensorMap tb = b_mn ? make_tmap_3d_bf16(w.data_ptr(), E, K, N, N, K * N, 64, 64)
                        : make_tmap_3d_bf16(w.data_ptr(), E, N, K, K, K * N, 64, pair ? 128 : 256);
  CUtensorMap to = make_tmap_bf16_epi(out.data_ptr(), out.size(0), N, out.stride(0));
  if (pair) {
    const int ub = (int)((a.size(0) / 256) * ((N + 255) / 256));
    const int grid = std::max(1, std::min(ub, num_pairs()));
    if (b_mn) launch<256, false, true, kGroupM, kStoreBF16, false, true>(ta, tb, args, grid, &to);
    else launch<256, false, false, kGroupM, kStoreBF16, false, true>(ta, tb, args, grid, &to);
    return;
  }
  const int ub = (int)((a.size(0) / BM) * ((N + 255) / 256));
  const int grid = std::max(1, std::min(ub, num_sms()));
  if (b_mn) launch<256, false, true, kGroupM, kStoreBF16, false>(ta, tb, args, grid, &to);
  else launch<256, false, false, kGroupM, kStoreBF16, false>(ta, tb, args, grid, &to);
}

}  // namespace pm

PM_DEFINE_ERROR_QUERY(pm_error_gemm_moe_fwd)
