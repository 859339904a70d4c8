// Validation kernel for the tcgen05 block-scaled MMA path: one CTA computes
// D[128, N] = A[128, K] * B[N, K]^T with e4m3 operands and UE8M0 scales per 32 K,
// everything staged through SMEM exactly as the production kernels do.
#include "tcgen05.cuh"
#include "torch_glue.h"

namespace moet {

__global__ void __launch_bounds__(128, 1) tc_gemm_test_kernel(const uint8_t* __restrict__ A, const uint8_t* __restrict__ SA,
                                                           const uint8_t* __restrict__ B, const uint8_t* __restrict__ SB,
                                                           int N, int K, float* __restrict__ out, int* status, int stage) {
  extern __shared__ __align__(1024) uint8_t sm[];
  uint8_t* sA = sm;                         // 128 x K
  uint8_t* sB = sA + 128 * K;               // N x K (N padded to 8)
  uint8_t* sSFA = sB + ((N + 7) / 8) * 8 * K;   // (K/128) x 512
  uint8_t* sSFB = sSFA + (K / 128) * 512;
  __shared__ uint64_t bar;
  __shared__ uint32_t taddr_s;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int KB = K / 32;
  for (int i = tid; i < 128 * K; i += blockDim.x) sA[tc::kmajor_off(i / K, i % K, K)] = A[i];
  for (int i = tid; i < N * K; i += blockDim.x) sB[tc::kmajor_off(i / K, i % K, K)] = B[i];
  for (int i = tid; i < (K / 128) * 512; i += blockDim.x) { sSFA[i] = 0; sSFB[i] = 0; }
  __syncthreads();
  for (int i = tid; i < 128 * KB; i += blockDim.x) sSFA[tc::sf_off(i / KB, i % KB)] = SA[i];
  for (int i = tid; i < N * KB; i += blockDim.x) sSFB[tc::sf_off(i / KB, i % KB)] = SB[i];
  if (warp == 0) tc::tmem_alloc(&taddr_s, 512);
  if (tid == 0) { tc::mbar_init(&bar, 1); }
  tc::fence_proxy_async_smem();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = taddr_s;
  const uint32_t t_d = tmem, t_sfa = tmem + 256, t_sfb = tmem + 256 + 64;
  bool ok = true;
  if (tid == 0 && stage >= 1) {
    for (int j = 0; j < K / 128; j++) {
      tc::cp_sf_32x128b_warpx4(t_sfa + 4 * j, tc::smem_desc(tc::smem_addr(sSFA + 512 * j), 0, 128));
      tc::cp_sf_32x128b_warpx4(t_sfb + 4 * j, tc::smem_desc(tc::smem_addr(sSFB + 512 * j), 0, 128));
    }
    const uint32_t sbo_a = (K / 16) * 128;
    for (int kb = 0; kb < KB && stage >= 2; kb++) {
      const uint64_t da = tc::smem_desc(tc::smem_addr(sA + kb * 256), 128, sbo_a);
      const uint64_t db = tc::smem_desc(tc::smem_addr(sB + kb * 256), 128, sbo_a);
      tc::mma_mxf8(t_d, da, db, tc::idesc_mxf8(128, (N + 7) / 8 * 8, kb & 3, kb & 3), kb > 0,
                   t_sfa + (kb >> 2) * 4, t_sfb + (kb >> 2) * 4);
    }
    tc::commit(&bar);
  }
  if (stage >= 1) ok = tc::mbar_wait(&bar, 0);
  if (!ok && tid == 0) set_status(status, kTimeout);
  tc::fence_after();
  if (ok && stage >= 3) {
    // warp w reads lanes [32w, 32w+32): row = 32w + lane
    const int row = warp * 32 + (tid & 31);
    for (int c0 = 0; c0 < N; c0 += 8) {
      uint32_t r[8];
      tc::tmem_ld8(tmem + ((uint32_t)(warp * 32) << 16) + c0, r);
      tc::tmem_wait_ld();
      for (int j = 0; j < 8 && c0 + j < N; j++) out[(size_t)(c0 + j) * 128 + row] = __uint_as_float(r[j]);
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) { tc::tmem_dealloc(tmem, 512); tc::tmem_relinquish(); }
}

}  // namespace moet

using namespace moet;

// a [128, K] e4m3 bytes, sa [128, K/32] ue8m0, b [N, K], sb [N, K/32]; out [N, 128] f32
void tc_gemm_test(torch::Tensor a, torch::Tensor sa, torch::Tensor b, torch::Tensor sb, torch::Tensor out,
                  torch::Tensor status, int64_t stage) {
  const int K = a.size(1), N = b.size(0);
  TORCH_CHECK(a.size(0) == 128 && K % 128 == 0 && K <= 512 && N >= 1 && N <= 128, "tc_gemm_test shape (one 128-row scale atom: N <= 128)");
  const size_t smem = 128 * K + ((N + 7) / 8) * 8 * K + 2 * (K / 128) * 512;
  TORCH_CHECK(smem <= 200 * 1024, "tc_gemm_test: smem");
  moet_allow_max_smem(tc_gemm_test_kernel);
  auto stream = at::cuda::getCurrentCUDAStream();
  tc_gemm_test_kernel<<<1, 128, smem, stream>>>((const uint8_t*)a.data_ptr(), (const uint8_t*)sa.data_ptr(),
                                                (const uint8_t*)b.data_ptr(), (const uint8_t*)sb.data_ptr(), N, K,
                                                out.data_ptr<float>(), status.data_ptr<int>(), (int)stage);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
