// tcgen05 GEMM entry points: expert fc2 dgrad + dSwiGLU, expert weight gradients.
// The kernel template, tile scheduler and epilogues are in gemm_sm100.cuh.
#include "gemm_sm100.cuh"

namespace pm {

// Expert fc2 data gradient fused with the SwiGLU backward:
//   dh_raw = dy[rows, H] . W2[e]  (W2: [E, H, I])
//   dgu[rows, 2I] = d(gate|up) of h = scale * silu(g) * u, using the saved gu
//   dscale[row] += sum_j silu(g) u dh_raw
void moe_fc2_dgrad_dswiglu(torch::Tensor dy, torch::Tensor w2, torch::Tensor offsets, torch::Tensor gu,
                           torch::Tensor scale, torch::Tensor dgu, torch::Tensor dscale, int64_t align) {
  TORCH_CHECK(align == 128 || align == 256, "segment alignment must be 128 or 256");
  check_bf16_2d(dy, "dy");
  check_bf16_2d(gu, "gu");
  check_bf16_2d(dgu, "dgu");
  TORCH_CHECK(w2.dim() == 3 && w2.is_contiguous() && w2.scalar_type() == torch::kBFloat16, "w2 must be [E,H,I]");
  const int64_t E = w2.size(0), H = w2.size(1), I = w2.size(2);
  TORCH_CHECK(dy.size(1) == H && gu.size(1) == 2 * I && dgu.size(1) == 2 * I, "shape mismatch");
  TORCH_CHECK(I % 128 == 0, "moe intermediate size must be a multiple of 128");
  TORCH_CHECK(scale.scalar_type() == torch::kFloat32 && dscale.scalar_type() == torch::kFloat32, "fp32 scales");
  PM_CHECK_CUDA(w2); PM_CHECK_CUDA(offsets); PM_CHECK_CUDA(scale); PM_CHECK_CUDA(dscale);
  TORCH_CHECK(offsets.numel() == E + 1 && offsets.scalar_type() == torch::kInt32, "offsets");
  c10::cuda::CUDAGuard guard(dy.device());
  GemmArgs args = blank_args();
  args.M = (int)dy.size(0); args.N = (int)I; args.K = (int)H; args.num_groups = (int)E;
  args.group_offsets = offsets.data_ptr<int>();
  args.raster = 1;  // an expert's weights (<= tens of MB) stay in L2 while its rows stream once
  args.row_scale = scale.data_ptr<float>();
  args.aux = reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()); args.ld_aux = gu.stride(0);
  args.aux_out = reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr()); args.ld_aux_out = dgu.stride(0);
  args.row_grad = dscale.data_ptr<float>();
  args.inter = (int)I;
  CUtensorMap ta = make_tmap_2d_bf16(dy.data_ptr(), dy.size(0), H, dy.stride(0), 64, 128);
  CUtensorMap tb = make_tmap_3d_bf16(w2.data_ptr(), E, H, I, I, H * I, 64, 64);
  // saved activations in, d(gate|up) out: 32 x 32 epilogue boxes
  CUtensorMap tg = make_tmap_bf16_epi(gu.data_ptr(), gu.size(0), 2 * I, gu.stride(0));
  CUtensorMap tdg = make_tmap_bf16_epi(dgu.data_ptr(), dgu.size(0), 2 * I, dgu.stride(0));
  if (align == 256) {
    if (I % 256 == 0) {
      const int ub = (int)((dy.size(0) / 256) * (I / 256));
      launch<256, false, true, kGroupM, kDSwiGLU, false, true>(ta, tb, args, std::max(1, std::min(ub, num_pairs())),
                                                               &tg, &tdg);
    } else {
      const int ub = (int)((dy.size(0) / 256) * (I / 128));
      launch<128, false, true, kGroupM, kDSwiGLU, false, true>(ta, tb, args, std::max(1, std::min(ub, num_pairs())),
                                                               &tg, &tdg);
    }
  } else if (I % 256 == 0) {
    const int ub = (int)((dy.size(0) / BM) * (I / 256));
    launch<256, false, true, kGroupM, kDSwiGLU, false>(ta, tb, args, std::max(1, std::min(ub, num_sms())), &tg, &tdg);
  } else {
    const int ub = (int)((dy.size(0) / BM) * (I / 128));
    launch<128, false, true, kGroupM, kDSwiGLU, false>(ta, tb, args, std::max(1, std::min(ub, num_sms())), &tg, &tdg);
  }
}

// Expert weight gradient: dw[e] (+)= a[seg_e]^T . b[seg_e]
//   a: [rows, M] (e.g. dY), b: [rows, N] (e.g. h); dw: [E, M, N] fp32.
//   gather_idx (optional, int32 [rows]): row r of b is b[gather_idx[r]] (TMA row gathers).
void moe_wgrad(torch::Tensor a, torch::Tensor b, torch::Tensor offsets, torch::Tensor dw, bool accumulate,
               c10::optional<torch::Tensor> gather_idx) {
  const bool gather = gather_idx.has_value();
  if (gather) {
    TORCH_CHECK(gather_idx->is_cuda() && gather_idx->scalar_type() == torch::kInt32 && gather_idx->is_contiguous(),
                "gather_idx must be a contiguous int32 CUDA tensor");
    TORCH_CHECK(gather_idx->numel() == a.size(0), "gather_idx must have one entry per row of a");
    TORCH_CHECK((reinterpret_cast<uintptr_t>(gather_idx->data_ptr()) & 15) == 0, "gather_idx must be 16-byte aligned");
  }
  check_bf16_2d(a, "a");
  check_bf16_2d(b, "b");
  TORCH_CHECK(dw.dim() == 3 && dw.is_contiguous() && dw.scalar_type() == torch::kFloat32, "dw must be fp32 [E,M,N]");
  const int64_t E = dw.size(0), M = dw.size(1), N = dw.size(2);
  TORCH_CHECK(a.size(1) == M && b.size(1) == N && (gather || a.size(0) == b.size(0)), "shape mismatch");
  TORCH_CHECK(M % 128 == 0 && N % 8 == 0, "M must be a multiple of 128");
  TORCH_CHECK(E <= kMaxGroups && offsets.numel() == E + 1 && offsets.scalar_type() == torch::kInt32, "offsets");
  PM_CHECK_CUDA(dw); PM_CHECK_CUDA(offsets);
  c10::cuda::CUDAGuard guard(a.device());
  GemmArgs args = blank_args();
  args.M = (int)M; args.N = (int)N; args.K = (int)a.size(0); args.num_groups = (int)E;
  args.group_offsets = offsets.data_ptr<int>();
  args.D = dw.data_ptr(); args.ldd = N; args.d_group_stride = M * N;
  args.beta = accumulate ? 1.f : 0.f;
  if (gather) args.gather_idx = gather_idx->data_ptr<int>();
  CUtensorMap ta = make_tmap_2d_bf16(a.data_ptr(), a.size(0), M, a.stride(0), 64, 64);
  CUtensorMap tb = make_tmap_2d_bf16(b.data_ptr(), b.size(0), N, b.stride(0), 64, gather ? 1 : 64);
  CUtensorMap td = make_tmap_f32_out(dw.data_ptr(), E, M, N, N, M * N, true);
  if (M % 256 == 0) {  // CTA pairs over 256 output rows
    const int tiles = (int)(E * (M / 256) * ((N + 255) / 256));
    if (gather) launch<256, true, true, kGroupK, kAccumF32, false, true, true>(ta, tb, args, std::min(tiles, num_pairs()), &td);
    else launch<256, true, true, kGroupK, kAccumF32, false, true>(ta, tb, args, std::min(tiles, num_pairs()), &td);
    return;
  }
  const int tiles = (int)(E * (M / BM) * ((N + 255) / 256));
  if (gather) launch<256, true, true, kGroupK, kAccumF32, false, false, true>(ta, tb, args, std::min(tiles, num_sms()), &td);
  else launch<256, true, true, kGroupK, kAccumF32, false>(ta, tb, args, std::min(tiles, num_sms()), &td);
}

}  // namespace pm

PM_DEFINE_ERROR_QUERY(pm_error_gemm_moe_bwd)
