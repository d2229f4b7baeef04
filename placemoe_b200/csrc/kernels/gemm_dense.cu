// tcgen05 GEMM entry points: dense layouts (forward, data gradient, weight gradient).
// The kernel template, tile scheduler and epilogues are in gemm_sm100.cuh.
#include "gemm_sm100.cuh"

namespace pm {

// out[M, N] (bf16 or fp32) = A . B^T with the layouts described at the top.
// accumulate: only for fp32 outputs (out += result).
void dense_gemm(torch::Tensor a, torch::Tensor b, torch::Tensor out, bool a_mn, bool b_mn, bool accumulate) {
  check_bf16_2d(a, "a");
  check_bf16_2d(b, "b");
  TORCH_CHECK(out.is_cuda() && out.dim() == 2 && out.stride(1) == 1, "out must be a 2-D CUDA tensor");
  const int64_t M = a_mn ? a.size(1) : a.size(0);
  const int64_t K = a_mn ? a.size(0) : a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  const int64_t Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "contraction sizes differ: ", K, " vs ", Kb);
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "out has the wrong shape");
  TORCH_CHECK(N % 8 == 0, "N must be a multiple of 8");
  if (M == 0 || N == 0) return;
  const bool f32 = out.scalar_type() == torch::kFloat32;
  TORCH_CHECK(f32 || out.scalar_type() == torch::kBFloat16, "out must be bf16 or fp32");
  TORCH_CHECK(!accumulate || f32, "accumulate requires an fp32 output");
  c10::cuda::CUDAGuard guard(a.device());
  if (K == 0) {
    if (!accumulate) out.zero_();
    return;
  }
  GemmArgs args = blank_args();
  args.M = (int)M; args.N = (int)N; args.K = (int)K;
  args.D = out.data_ptr(); args.ldd = out.stride(0); args.beta = accumulate ? 1.f : 0.f;
  // keep the smaller operand resident in L2 and stream the larger one once
  args.raster = M > N ? 1 : 0;

  // BN = 64 for narrow outputs (router logits), 256 otherwise.
  const bool narrow = N <= 64;
  const int BN = narrow ? 64 : 256;
  CUtensorMap ta = a_mn ? make_tmap_2d_bf16(a.data_ptr(), K, M, a.stride(0), 64, 64)
                        : make_tmap_2d_bf16(a.data_ptr(), M, K, a.stride(0), 64, 128);
  // CTA pairs (256-row tiles) once M fills them
  const bool pair = !narrow && M >= 256;
  CUtensorMap tb = b_mn ? make_tmap_2d_bf16(b.data_ptr(), K, N, b.stride(0), 64, 64)
                        : make_tmap_2d_bf16(b.data_ptr(), N, K, b.stride(0), 64, pair ? BN / 2 : BN);
  const int tiles = (int)(((M + BM - 1) / BM) * ((N + BN - 1) / BN));
  const int grid = std::min(tiles, num_sms());
  // bf16 results leave through TMA stores of 32 x 32 boxes
  CUtensorMap to;
  if (!f32) {
    TORCH_CHECK((out.stride(0) * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0,
                "bf16 output rows must be 16-byte aligned");
    to = make_tmap_bf16_epi(out.data_ptr(), M, N, out.stride(0));
  }
  if (pair) {
    const int ptiles = (int)(((M + 255) / 256) * ((N + BN - 1) / BN));
    const int pgrid = std::min(ptiles, num_pairs());
    if (!a_mn && !b_mn) {
      if (f32) launch<256, false, false, kGroupNone, kStoreF32, false, true>(ta, tb, args, pgrid);
      else launch<256, false, false, kGroupNone, kStoreBF16, false, true>(ta, tb, args, pgrid, &to);
    } else if (!a_mn && b_mn) {
      TORCH_CHECK(!f32, "dgrad layout produces bf16");
      launch<256, false, true, kGroupNone, kStoreBF16, false, true>(ta, tb, args, pgrid, &to);
    } else if (a_mn && b_mn) {
      if (f32) {
        TORCH_CHECK(N % 4 == 0 && (out.stride(0) % 4) == 0, "fp32 weight-gradient output needs N % 4 == 0");
        CUtensorMap td = make_tmap_f32_out(out.data_ptr(), 1, M, N, out.stride(0), 0, false);
        launch<256, true, true, kGroupNone, kAccumF32, false, true>(ta, tb, args, pgrid, &td);
      } else {
        launch<256, true, true, kGroupNone, kStoreBF16, false, true>(ta, tb, args, pgrid, &to);
      }
    } else {
      TORCH_CHECK(false, "unsupported layout combination (a MN-major with b K-major)");
    }
    return;
  }
  if (narrow) {
    TORCH_CHECK(!a_mn && !b_mn, "narrow GEMM supports the forward layout only");
    if (f32) launch<64, false, false, kGroupNone, kStoreF32, false>(ta, tb, args, grid);
    else launch<64, false, false, kGroupNone, kStoreBF16, false>(ta, tb, args, grid, &to);
    return;
  }
  if (!a_mn && !b_mn) {
    if (f32) launch<256, false, false, kGroupNone, kStoreF32, false>(ta, tb, args, grid);
    else launch<256, false, false, kGroupNone, kStoreBF16, false>(ta, tb, args, grid, &to);
  } else if (!a_mn && b_mn) {
    TORCH_CHECK(!f32, "dgrad layout produces bf16");
    launch<256, false, true, kGroupNone, kStoreBF16, false>(ta, tb, args, grid, &to);
  } else if (a_mn && b_mn) {
    if (f32) {
      TORCH_CHECK(N % 4 == 0 && (out.stride(0) % 4) == 0, "fp32 weight-gradient output needs N % 4 == 0");
      CUtensorMap td = make_tmap_f32_out(out.data_ptr(), 1, M, N, out.stride(0), 0, false);
      launch<256, true, true, kGroupNone, kAccumF32, false>(ta, tb, args, grid, &td);
    }
    else launch<256, true, true, kGroupNone, kStoreBF16, false>(ta, tb, args, grid, &to);
  } else {
    TORCH_CHECK(false, "unsupported layout combination (a MN-major with b K-major)");
  }
}

}  // namespace pm

PM_DEFINE_ERROR_QUERY(pm_error_gemm_dense)
