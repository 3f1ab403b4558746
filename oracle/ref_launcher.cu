// C launcher for the reference's own CUDA kernels (TEST INFRASTRUCTURE: used
// only by GPU cross-check tests and bench comparators, never by the product).
//
// Compiled by oracle/Makefile together with the reference's gemm.cu, which is
// #included from where it lies in the reference tree (-I points there); no
// reference source is copied into this repository.  The launch geometry and
// shared-memory sizes restate the reference launcher (tensorcore_gemm/gemm.py
// :53-148): 256 x 128 x 32 tiles, 3 stages, padding 8, 256 threads, grid
// (16, ceil(M/256), ceil(ceil(N/128)/16)), alpha = 1, beta = 0.  Like the
// reference it requires M % 256 == 0, N % 128 == 0, K % 32 == 0, K >= 64
// (gemm.py:185-192); this launcher refuses other shapes instead of running
// them out of bounds.
#include "gemm.cu"

namespace {
constexpr int kTileM = 256, kTileN = 128, kKTile = 32, kPad = 8, kStages = 3, kThreads = 256;

template <typename Kern>
int launch(Kern kern, int smem, const half* A, const half* B, half* C, int M, int N, int K, cudaStream_t s) {
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return 4;
  dim3 grid(16, (M + kTileM - 1) / kTileM, ((N + kTileN - 1) / kTileN + 16 - 1) / 16);
  kern<<<grid, kThreads, smem, s>>>(A, B, C, M, N, K, 1.0f, 0.0f);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}
}  // namespace

// mode: 2 reg_pingpong_256, 3 reg_pingpong_256_mma (B row-major K x N);
//       4 reg_pingpong_256_colb, 5 reg_pingpong_256_colb_mma (B stored N x K).
// Returns 0 on success, 1 bad argument / unsupported shape, 4 CUDA error.
extern "C" __attribute__((visibility("default"))) int ref_gemm_launch(const void* A, const void* B, void* C, int M,
                                                                      int N, int K, int mode, void* stream) {
  if (!A || !B || !C || M <= 0 || N <= 0 || K < 64) return 1;
  if (M % kTileM || N % kTileN || K % kKTile) return 1;
  const half* a = static_cast<const half*>(A);
  const half* b = static_cast<const half*>(B);
  half* c = static_cast<half*>(C);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int smem_rowb = kStages * (kTileM * (kKTile + kPad) + kKTile * (kTileN + kPad)) * 2;
  const int smem_colb = kStages * (kTileM * (kKTile + kPad) + kTileN * (kKTile + kPad)) * 2;
  const int smem_mma = smem_colb + (kKTile * (kTileN + kPad)) * 2;
  switch (mode) {
    case 2: return launch(gemm_3_stage_buffer_kernel_32_swizzled_rotate3_reg_pingpong_256, smem_rowb, a, b, c, M, N, K, s);
    case 3: return launch(gemm_3_stage_buffer_kernel_32_swizzled_rotate3_reg_pingpong_256_MMA, smem_mma, a, b, c, M, N, K, s);
    case 4: return launch(gemm_3_stage_buffer_kernel_32_swizzled_rotate3_reg_pingpong_256_colb, smem_colb, a, b, c, M, N, K, s);
    case 5: return launch(gemm_3_stage_buffer_kernel_32_swizzled_rotate3_reg_pingpong_256_colb_MMA, smem_colb, a, b, c, M, N, K, s);
    default: return 1;
  }
}
