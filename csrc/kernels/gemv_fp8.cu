// Skinny FP8 GEMM for decode ("weight-streaming GEMV"): out[T, N] = A[T, K] * W[N, K]^T
// with W e4m3 row-major + UE8M0 128x128 block scales and A e4m3 (natural
// layout) + UE8M0 per-64 scales.  T is small (1..128 tokens): the kernel
// streams W once from HBM at full width (16 B per lane per row per 64-k
// chunk) and reuses each weight fragment for every n8 token tile.
//
// One CTA owns 16 output rows; its warps split K by 64-wide chunks
// round-robin and reduce through shared memory.  The MMA is
// mma.sync m16n8k32 e4m3 with the weight rows as the M=16 operand
// ("swap-AB"); a consistent permutation of k inside each 64-chunk lets
// every lane issue one 16-byte load per row and per token:
//   lane (g,t) loads W[row g / g+8][c*64 + 16t .. +15] and A[tok g][same]
//   MMA 0 uses bytes 0..7, MMA 1 bytes 8..15.
// Optional batch dimension (blockIdx.z) for per-head weights (MLA absorb).
#include "common.cuh"
#include "symm.cuh"
#include "torch_glue.h"

namespace moet {

struct GemvArgs {
  const uint8_t* A; const uint8_t* sA; const uint8_t* W; const uint8_t* sW;
  void* out; const __nv_bfloat16* resid;
  int T, N, K;
  long long a_row_stride, a_batch_stride;     // bytes / elements (e4m3 = 1 byte)
  long long sa_row_stride, sa_batch_stride;   // bytes
  long long w_batch_stride, sw_batch_stride;  // bytes
  long long out_row_stride, out_batch_stride; // elements
  int sw_cols;                                // K/128 (ceil)
  int out_f32;
  int ar_on;                                  // push fp32 partials to every TP peer instead of writing out
  ArDesc ar;
};

template <int NT>
__global__ void __launch_bounds__(256) gemv_fp8_kernel(GemvArgs p) {
  extern __shared__ float red[];  // [nwarps][NT*4][32]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int nwarps = blockDim.x >> 5;
  const int row0 = blockIdx.x * 16;
  const int tok0 = blockIdx.y * 8 * NT;
  const int b = blockIdx.z;
  if (blockIdx.y == 0) {   // weights are immutable: pull this CTA's rows toward L2 while the previous kernel runs
    const int lines = p.K >> 7, nrows = min(16, p.N - row0);
    const uint8_t* wbase = p.W + (size_t)b * p.w_batch_stride + (size_t)row0 * p.K;
    for (int i = threadIdx.x; i < nrows * lines; i += blockDim.x) prefetch_l2(wbase + (size_t)i * 128);
  }
  pdl_entry();
  const uint8_t* A = p.A + (size_t)b * p.a_batch_stride;
  const uint8_t* sA = p.sA + (size_t)b * p.sa_batch_stride;
  const uint8_t* W = p.W + (size_t)b * p.w_batch_stride;
  const uint8_t* sW = p.sW + (size_t)b * p.sw_batch_stride;
  const int ra = min(row0 + g, p.N - 1), rb = min(row0 + g + 8, p.N - 1);
  const uint8_t* wa_p = W + (size_t)ra * p.K + 16 * t;
  const uint8_t* wb_p = W + (size_t)rb * p.K + 16 * t;
  const uint8_t* sw_row = sW + (size_t)(row0 >> 7) * p.sw_cols;
  const int nchunks = p.K >> 6;

  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

  // token rows this lane feeds as the B operand (column g of each n8 tile)
  const uint8_t* xbase = A + 16 * t;
  const int tg = tok0 + g, tc = tok0 + 2 * t;

  // Each warp takes U consecutive chunks per step and issues all of their weight
  // loads before consuming any, keeping U * 1 KiB per warp in flight.
  constexpr int U = NT <= 1 ? 8 : (NT <= 2 ? 4 : 2);
  for (int cb = warp * U; cb < nchunks; cb += nwarps * U) {
    uint4 wa[U], wb[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      if (cb + u < nchunks) {
        wa[u] = ldg_stream_u4(wa_p + (size_t)(cb + u) * 64);
        wb[u] = ldg_stream_u4(wb_p + (size_t)(cb + u) * 64);
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int c = cb + u;
      if (c >= nchunks) break;
      const float ws = ue8m0_to_float(sw_row[c >> 1]);
      const uint32_t a0[4] = {wa[u].x, wb[u].x, wa[u].y, wb[u].y};
      const uint32_t a1[4] = {wa[u].z, wb[u].z, wa[u].w, wb[u].w};
#pragma unroll
      for (int nt = 0; nt < NT; nt++) {
        uint4 x = make_uint4(0, 0, 0, 0);
        const int tok = tg + nt * 8;
        if (tok < p.T) x = __ldg(reinterpret_cast<const uint4*>(xbase + (size_t)tok * p.a_row_stride + (size_t)c * 64));
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        mma_e4m3_16832(d, a0, x.x, x.y, d);
        mma_e4m3_16832(d, a1, x.z, x.w, d);
        const int c0 = tc + nt * 8;
        const float s0 = c0 < p.T ? ws * ue8m0_to_float(sA[(size_t)c0 * p.sa_row_stride + c]) : 0.f;
        const float s1 = c0 + 1 < p.T ? ws * ue8m0_to_float(sA[(size_t)(c0 + 1) * p.sa_row_stride + c]) : 0.f;
        acc[nt][0] = fmaf(d[0], s0, acc[nt][0]);
        acc[nt][1] = fmaf(d[1], s1, acc[nt][1]);
        acc[nt][2] = fmaf(d[2], s0, acc[nt][2]);
        acc[nt][3] = fmaf(d[3], s1, acc[nt][3]);
      }
    }
  }

  // cross-warp reduction
  if (nwarps > 1) {
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int i = 0; i < 4; i++) red[((warp * NT + nt) * 4 + i) * 32 + lane] = acc[nt][i];
    __syncthreads();
    if (warp != 0) return;
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        float s = 0.f;
        for (int w = 0; w < nwarps; w++) s += red[((w * NT + nt) * 4 + i) * 32 + lane];
        acc[nt][i] = s;
      }
  }

  if (p.ar_on) {   // row-parallel GEMV -> all-reduce: push this tile into slot [rank] of every peer
    const unsigned long long epoch = ar_epoch(p.ar);
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int row = row0 + g + ((i & 2) ? 8 : 0);
        const int tok = tok0 + nt * 8 + 2 * t + (i & 1);
        if (row >= p.N || tok >= p.T) continue;
        const size_t off = (size_t)tok * p.N + row;
        for (int q = 0; q < p.ar.world; q++) ar_slot(p.ar, q, epoch, p.ar.rank)[off] = acc[nt][i];
      }
    ar_producer_arrive(p.ar, epoch, /*warp_only=*/true);
    return;
  }
  char* outb = reinterpret_cast<char*>(p.out);
  const size_t esz = p.out_f32 ? 4 : 2;
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int row = row0 + g + ((i & 2) ? 8 : 0);
      const int tok = tok0 + nt * 8 + 2 * t + (i & 1);
      if (row >= p.N || tok >= p.T) continue;
      const size_t off = (size_t)b * p.out_batch_stride + (size_t)tok * p.out_row_stride + row;
      float v = acc[nt][i];
      if (p.resid) v += __bfloat162float(p.resid[(size_t)tok * p.out_row_stride + row]);
      if (p.out_f32) reinterpret_cast<float*>(outb)[off] = v;
      else reinterpret_cast<__nv_bfloat16*>(outb)[off] = __float2bfloat16(v);
    }
  (void)esz;
}

}  // namespace moet

using namespace moet;

// a: [B?, T, K] u8 (row stride in bytes = a.stride(-2)); sa: [B?, T, K/64];
// w: [B?, N, K] u8; sw: [B?, ceil(N/128), ceil(K/128)]; out: [B?, T, N] bf16|f32.
void gemv_fp8(torch::Tensor a, torch::Tensor sa, torch::Tensor w, torch::Tensor sw, torch::Tensor out,
              c10::optional<torch::Tensor> resid, c10::optional<torch::Tensor> ar) {
  const bool batched = w.dim() == 3;
  const int B = batched ? w.size(0) : 1;
  const int N = w.size(-2), K = w.size(-1);
  const int T = a.size(-2);
  TORCH_CHECK(K % 64 == 0, "gemv_fp8: K must be a multiple of 64");
  TORCH_CHECK(a.size(-1) == K, "gemv_fp8: A/W K mismatch");
  TORCH_CHECK(w.stride(-1) == 1 && w.stride(-2) == K, "gemv_fp8: W must be row-major contiguous per batch");
  TORCH_CHECK(a.stride(-1) == 1 && sa.stride(-1) == 1 && out.stride(-1) == 1, "gemv_fp8: inner strides must be 1");
  TORCH_CHECK(sw.size(-1) == (K + 127) / 128 && sw.size(-2) == (N + 127) / 128, "gemv_fp8: weight scale shape");
  TORCH_CHECK(a.data_ptr() != nullptr && reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0 &&
                  a.stride(-2) % 16 == 0, "gemv_fp8: A rows must be 16-byte aligned");
  if (T == 0) return;
  GemvArgs p;
  p.A = (const uint8_t*)a.data_ptr(); p.sA = (const uint8_t*)sa.data_ptr();
  p.W = (const uint8_t*)w.data_ptr(); p.sW = (const uint8_t*)sw.data_ptr();
  p.out = out.data_ptr();
  p.resid = resid.has_value() && resid->defined() ? (const __nv_bfloat16*)resid->data_ptr() : nullptr;
  if (p.resid) TORCH_CHECK(!batched && resid->stride(0) == out.stride(0), "gemv_fp8: resid layout");
  p.T = T; p.N = N; p.K = K;
  p.a_row_stride = a.stride(-2); p.a_batch_stride = batched ? a.stride(0) : 0;
  p.sa_row_stride = sa.stride(-2); p.sa_batch_stride = batched ? sa.stride(0) : 0;
  p.w_batch_stride = batched ? w.stride(0) : 0; p.sw_batch_stride = batched ? sw.stride(0) : 0;
  p.out_row_stride = out.stride(-2); p.out_batch_stride = batched ? out.stride(0) : 0;
  p.sw_cols = sw.size(-1);
  p.out_f32 = out.scalar_type() == at::kFloat;
  p.ar_on = ar.has_value() && ar->defined();
  if (p.ar_on) {
    p.ar = ar_desc_from(*ar);
    TORCH_CHECK(!batched && !p.resid && (int64_t)T * N <= p.ar.cap, "gemv_fp8: all-reduce push needs an unbatched GEMV, "
                "no residual and T*N <= the slot capacity");
  }
  TORCH_CHECK(p.out_f32 || out.scalar_type() == at::kBFloat16, "gemv_fp8: out must be bf16 or f32");
  const int nchunks = K / 64;
  auto stream = at::cuda::getCurrentCUDAStream();
  auto launch = [&](auto nt_const) {
    constexpr int NT = decltype(nt_const)::value;
    constexpr int U = NT <= 1 ? 8 : (NT <= 2 ? 4 : 2);
    const int nwarps = std::max(1, std::min(8, (nchunks + U - 1) / U));
    dim3 grid((N + 15) / 16, (T + 8 * NT - 1) / (8 * NT), B);
    size_t smem = nwarps > 1 ? (size_t)nwarps * NT * 4 * 32 * sizeof(float) : 0;
    if (smem > 48 * 1024) moet_allow_max_smem(gemv_fp8_kernel<NT>);
    cudaFuncSetAttribute(gemv_fp8_kernel<NT>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    launch_k(gemv_fp8_kernel<NT>, grid, nwarps * 32, smem, stream, p);
  };
  if (T <= 8) launch(std::integral_constant<int, 1>{});
  else if (T <= 16) launch(std::integral_constant<int, 2>{});
  else if (T <= 32) launch(std::integral_constant<int, 4>{});
  else if (T <= 64) launch(std::integral_constant<int, 8>{});
  else launch(std::integral_constant<int, 16>{});
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
