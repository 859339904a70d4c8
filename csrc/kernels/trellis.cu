// Trellis-coded (EXL3-style) routed experts: the decode kernels of the trellis base tier.
//
// Format (vllm_moet_b200/formats/trellis.py): a linear y = x W^T is stored as
// W^T = diag(su) Hk Q Hn diag(sv), Hk / Hn block Walsh-Hadamard (block hb <= 128), su / sv
// fp16, Q [Kin, N] in 16 x 16 tiles ((k-tile, n-tile) row-major, value i = kk*16 + nn
// inside a tile).  A tile is one tail-biting bitshift trellis walk of 256*KB bits in 16*KB
// 16-bit words (stream bit 0 = MSB of word 0); value i is cb(state_i) * inv_rms with
// state_i the L-bit window ending at stream bit (i + 1)*KB, read cyclically.  Codebooks
// from QTIP (Tseng et al., NeurIPS 2024): 3INST and 1MAD.  The reference serves this
// family of formats through exllamav3's exl3_mgemm and its M=8 decode-wave cubins
// (patch/vllm-moet-v0.24.0.patch:10624-10700, kernels/MANIFEST.md:198-228); these
// kernels are our own.
//
// Three kernels per projection of a decode step over P = T*k routing pairs:
//   trellis_rot_in   grid P: x'[p] = H(x[src[p]] * su[eid[p]])       (smem butterfly)
//   trellis_gemv     grid (N/16/TN, G): group g = one expert and up to 8 pairs; every
//                    tile of the expert is decoded ONCE for all of the group's rows.  A
//                    warp walks the k-tiles of one n-tile; lane = (kk = lane/2, 8 columns
//                    nn0 = (lane&1)*8): the tile's words sit one per lane (two for KB > 2)
//                    and a lane assembles the 64 stream bits its 8 windows need from four
//                    shuffled words.  Lanes and then warps are summed in a fixed order.
//   trellis_rot_out  grid P: y[p] = H(z[p]) * sv[eid[p]] * (scale[p] or 1)
// No spin waits, no asynchronous copies; everything stays inside the launch.
#include "common.cuh"
#include "torch_glue.h"

#include <cuda_fp16.h>

namespace moet {

constexpr int kTrGemvWarps = 8;
constexpr int kTrTilesPerCta = 4;       // n-tiles (16 columns each) per trellis_gemv CTA
constexpr int kTrRotThreads = 256;

MOET_DEVICE float trellis_value(uint32_t s, bool mad, float scale) {
  if (!mad) {                                   // 3INST
    const uint32_t x = s * 89226354u + 64248484u;
    const uint32_t m = (x & 0x8FFF8FFFu) ^ 0x3B603B60u;
    const float lo = __half2float(__ushort_as_half((unsigned short)(m & 0xFFFFu)));
    const float hi = __half2float(__ushort_as_half((unsigned short)(m >> 16)));
    return (lo + hi) * scale;
  }
  const uint32_t x = s * 34038481u + 76625530u;   // 1MAD
  const int tot = (int)(x & 0xFFu) + (int)((x >> 8) & 0xFFu) + (int)((x >> 16) & 0xFFu) + (int)(x >> 24);
  return (float)(tot - 510) * scale;            // scale = inv_rms / 147.8 (host)
}

// in-place orthonormal block Walsh-Hadamard transform of n values in shared memory
MOET_DEVICE void fwht_smem(float* sm, int n, int hb) {
  for (int h = 1; h < hb; h <<= 1) {
    for (int j = threadIdx.x; j < n / 2; j += blockDim.x) {
      const int i0 = (j / h) * 2 * h + (j % h), i1 = i0 + h;
      const float a = sm[i0], c = sm[i1];
      sm[i0] = a + c;
      sm[i1] = a - c;
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kTrRotThreads) trellis_rot_in_kernel(
    const float* __restrict__ x, const int* __restrict__ src, const int* __restrict__ eid,
    const __half* __restrict__ su, float* __restrict__ out, int n, int hb, float norm) {
  extern __shared__ float tr_sm[];
  const int p = blockIdx.x, s = src[p], e = eid[p];
  float* o = out + (size_t)p * n;
  if (s < 0) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = 0.f;
    return;
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    tr_sm[i] = x[(size_t)s * n + i] * __half2float(su[(size_t)e * n + i]);
  __syncthreads();
  fwht_smem(tr_sm, n, hb);
  for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = tr_sm[i] * norm;
}

__global__ void __launch_bounds__(kTrRotThreads) trellis_rot_out_kernel(
    const float* __restrict__ z, const int* __restrict__ eid, const __half* __restrict__ sv,
    const float* __restrict__ scale, float* __restrict__ out, int n, int hb, float norm) {
  extern __shared__ float tr_sm[];
  const int p = blockIdx.x, e = eid[p];
  for (int i = threadIdx.x; i < n; i += blockDim.x) tr_sm[i] = z[(size_t)p * n + i];
  __syncthreads();
  fwht_smem(tr_sm, n, hb);
  const float w = (scale != nullptr ? scale[p] : 1.f) * norm;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    out[(size_t)p * n + i] = tr_sm[i] * w * __half2float(sv[(size_t)e * n + i]);
}

template <int MAXR, int KB>
__global__ void __launch_bounds__(kTrGemvWarps * 32) trellis_gemv_kernel(
    const float* __restrict__ xr, const uint16_t* __restrict__ trellis, const int* __restrict__ experts,
    const int* __restrict__ row_map, float* __restrict__ z, int Kt, int Nt, int L, bool mad, float scale) {
  constexpr int NW = 16 * KB;                   // words per tile
  constexpr int NBITS = 256 * KB;
  const int g = blockIdx.y;
  const int* rm = row_map + (size_t)g * 8;
  if (rm[0] < 0) return;                        // empty group (uniform over the CTA)
  const int e = experts[g];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Kin = Kt * 16, N = Nt * 16;
  int pr[MAXR];
#pragma unroll
  for (int r = 0; r < MAXR; r++) pr[r] = rm[r];
  __shared__ float red[kTrGemvWarps][MAXR][16];

  const int kk = lane >> 1, nn0 = (lane & 1) * 8;
  const int i0 = kk * 16 + nn0;
  int start = (i0 + 1) * KB - L;                // first bit of value i0's window (cyclic)
  if (start < 0) start += NBITS;
  const int w0 = start >> 4, sh = start & 15;
  const uint32_t smask = (1u << L) - 1u;

  const int nt_end = min(Nt, (int)(blockIdx.x + 1) * kTrTilesPerCta);
  for (int nt = blockIdx.x * kTrTilesPerCta; nt < nt_end; nt++) {
    float acc[MAXR][8];
#pragma unroll
    for (int r = 0; r < MAXR; r++)
#pragma unroll
      for (int j = 0; j < 8; j++) acc[r][j] = 0.f;
    for (int kt = warp; kt < Kt; kt += kTrGemvWarps) {
      const uint16_t* tile = trellis + (((size_t)e * Kt + kt) * Nt + nt) * NW;
      const uint32_t r0 = lane < NW ? tile[lane] : 0u;
      const uint32_t r1 = (NW > 32 && lane + 32 < NW) ? tile[lane + 32] : 0u;
      uint64_t u = 0;
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const int wi = (w0 + q) % NW;
        const uint32_t v0 = __shfl_sync(0xffffffffu, r0, wi & 31);
        const uint32_t v1 = __shfl_sync(0xffffffffu, r1, wi & 31);
        u = (u << 16) | (uint64_t)((wi >= 32 ? v1 : v0) & 0xFFFFu);
      }
      float xv[MAXR];
#pragma unroll
      for (int r = 0; r < MAXR; r++) xv[r] = pr[r] >= 0 ? __ldg(xr + (size_t)pr[r] * Kin + kt * 16 + kk) : 0.f;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const uint32_t s = (uint32_t)(u >> (64 - sh - j * KB - L)) & smask;
        const float qv = trellis_value(s, mad, scale);
#pragma unroll
        for (int r = 0; r < MAXR; r++) acc[r][j] = fmaf(xv[r], qv, acc[r][j]);
      }
    }
    // lanes of one column half (same lane & 1): fixed butterfly order
#pragma unroll
    for (int r = 0; r < MAXR; r++)
#pragma unroll
      for (int j = 0; j < 8; j++) {
        float v = acc[r][j];
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        acc[r][j] = v;
      }
    if (lane < 2) {
#pragma unroll
      for (int r = 0; r < MAXR; r++)
#pragma unroll
        for (int j = 0; j < 8; j++) red[warp][r][nn0 + j] = acc[r][j];
    }
    __syncthreads();
    if (threadIdx.x < MAXR * 16) {
      const int r = threadIdx.x / 16, c = threadIdx.x % 16;
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kTrGemvWarps; w++) s += red[w][r][c];
      const int pe = rm[r];
      if (pe >= 0) z[(size_t)pe * N + nt * 16 + c] = s;
    }
    __syncthreads();
  }
}

}  // namespace moet

using namespace moet;

static int tr_hadamard_block(int64_t n) {
  int b = 1;
  while (b < 128 && n % (2 * b) == 0) b *= 2;
  return b;
}

static void tr_check_pairs(const torch::Tensor& t, int64_t P, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kInt && t.dim() == 1 && t.size(0) == P && t.is_contiguous(),
              "trellis: ", name, " must be a contiguous int32 [P] CUDA tensor");
}

static void tr_rot_smem(int64_t n) {
  TORCH_CHECK(n % 2 == 0 && (size_t)n * sizeof(float) <= 200 * 1024, "trellis: rotation width ", n,
              " (needs an even width of at most 51200)");
}

void trellis_rot_in(torch::Tensor x, torch::Tensor src, torch::Tensor eid, torch::Tensor su, torch::Tensor out) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.dim() == 2 && x.is_contiguous(),
              "trellis_rot_in: x must be contiguous f32 [Tx, n]");
  TORCH_CHECK(su.is_cuda() && su.scalar_type() == at::kHalf && su.dim() == 2 && su.is_contiguous() &&
                  su.size(1) == x.size(1), "trellis_rot_in: su must be f16 [E, n]");
  const int64_t P = out.size(0), n = x.size(1);
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.dim() == 2 && out.size(1) == n &&
                  out.is_contiguous(), "trellis_rot_in: out must be contiguous f32 [P, n]");
  tr_check_pairs(src, P, "src");
  tr_check_pairs(eid, P, "eid");
  tr_rot_smem(n);
  if (P == 0) return;
  const int hb = tr_hadamard_block(n);
  const size_t smem = (size_t)n * sizeof(float);
  moet_allow_max_smem(trellis_rot_in_kernel);
  trellis_rot_in_kernel<<<(unsigned)P, kTrRotThreads, smem, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), src.data_ptr<int>(), eid.data_ptr<int>(),
      reinterpret_cast<const __half*>(su.data_ptr()), out.data_ptr<float>(), (int)n, hb, 1.f / sqrtf((float)hb));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void trellis_rot_out(torch::Tensor z, torch::Tensor eid, torch::Tensor sv, c10::optional<torch::Tensor> scale,
                     torch::Tensor out) {
  TORCH_CHECK(z.is_cuda() && z.scalar_type() == at::kFloat && z.dim() == 2 && z.is_contiguous(),
              "trellis_rot_out: z must be contiguous f32 [P, n]");
  const int64_t P = z.size(0), n = z.size(1);
  TORCH_CHECK(sv.is_cuda() && sv.scalar_type() == at::kHalf && sv.dim() == 2 && sv.is_contiguous() &&
                  sv.size(1) == n, "trellis_rot_out: sv must be f16 [E, n]");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.sizes() == z.sizes() && out.is_contiguous(),
              "trellis_rot_out: out must be contiguous f32 like z");
  tr_check_pairs(eid, P, "eid");
  if (scale.has_value())
    TORCH_CHECK(scale->is_cuda() && scale->scalar_type() == at::kFloat && scale->numel() == P &&
                    scale->is_contiguous(), "trellis_rot_out: scale must be contiguous f32 [P]");
  tr_rot_smem(n);
  if (P == 0) return;
  const int hb = tr_hadamard_block(n);
  const size_t smem = (size_t)n * sizeof(float);
  moet_allow_max_smem(trellis_rot_out_kernel);
  trellis_rot_out_kernel<<<(unsigned)P, kTrRotThreads, smem, at::cuda::getCurrentCUDAStream()>>>(
      z.data_ptr<float>(), eid.data_ptr<int>(), reinterpret_cast<const __half*>(sv.data_ptr()),
      scale.has_value() ? scale->data_ptr<float>() : nullptr, out.data_ptr<float>(), (int)n, hb,
      1.f / sqrtf((float)hb));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int MAXR>
static void tr_gemv_launch(dim3 grid, cudaStream_t st, int64_t K, const float* xr, const uint16_t* tr,
                           const int* ex, const int* rm, float* z, int Kt, int Nt, int L, bool mad, float scale) {
  const dim3 block(kTrGemvWarps * 32);
  switch (K) {
    case 1: trellis_gemv_kernel<MAXR, 1><<<grid, block, 0, st>>>(xr, tr, ex, rm, z, Kt, Nt, L, mad, scale); break;
    case 2: trellis_gemv_kernel<MAXR, 2><<<grid, block, 0, st>>>(xr, tr, ex, rm, z, Kt, Nt, L, mad, scale); break;
    case 3: trellis_gemv_kernel<MAXR, 3><<<grid, block, 0, st>>>(xr, tr, ex, rm, z, Kt, Nt, L, mad, scale); break;
    default: trellis_gemv_kernel<MAXR, 4><<<grid, block, 0, st>>>(xr, tr, ex, rm, z, Kt, Nt, L, mad, scale); break;
  }
}

void trellis_gemv(torch::Tensor xr, torch::Tensor trellis, torch::Tensor experts, torch::Tensor row_map,
                  torch::Tensor z, int64_t K, int64_t L, bool mad, double inv_rms, int64_t maxr) {
  TORCH_CHECK(K >= 1 && K <= 4 && L > K && L <= 16, "trellis_gemv: need 1 <= K <= 4 and K < L <= 16");
  TORCH_CHECK(trellis.is_cuda() && trellis.scalar_type() == at::kShort && trellis.dim() == 4 &&
                  trellis.size(3) == 16 * K && trellis.is_contiguous(),
              "trellis_gemv: trellis must be contiguous int16 [E, Kin/16, N/16, 16K]");
  const int64_t E = trellis.size(0), Kt = trellis.size(1), Nt = trellis.size(2);
  TORCH_CHECK(xr.is_cuda() && xr.scalar_type() == at::kFloat && xr.dim() == 2 && xr.size(1) == Kt * 16 &&
                  xr.is_contiguous(), "trellis_gemv: xr must be contiguous f32 [P, Kin]");
  const int64_t P = xr.size(0);
  TORCH_CHECK(z.is_cuda() && z.scalar_type() == at::kFloat && z.dim() == 2 && z.size(0) == P &&
                  z.size(1) == Nt * 16 && z.is_contiguous(), "trellis_gemv: z must be contiguous f32 [P, N]");
  TORCH_CHECK(row_map.is_cuda() && row_map.scalar_type() == at::kInt && row_map.dim() == 2 &&
                  row_map.size(1) == 8 && row_map.is_contiguous(), "trellis_gemv: row_map must be int32 [G, 8]");
  const int64_t G = row_map.size(0);
  TORCH_CHECK(experts.is_cuda() && experts.scalar_type() == at::kInt && experts.numel() == G &&
                  experts.is_contiguous(), "trellis_gemv: experts must be int32 [G]");
  TORCH_CHECK(maxr >= 1 && maxr <= 8, "trellis_gemv: rows per group 1..8");
  TORCH_CHECK(E < (1LL << 31) / 4 && Kt * Nt * 16 * K < (1LL << 40), "trellis_gemv: sizes");
  if (G == 0 || P == 0) return;
  const dim3 grid((unsigned)((Nt + kTrTilesPerCta - 1) / kTrTilesPerCta), (unsigned)G);
  const float scale = mad ? (float)(inv_rms / 147.8) : (float)inv_rms;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const float* xp = xr.data_ptr<float>();
  const uint16_t* tp = reinterpret_cast<const uint16_t*>(trellis.data_ptr());
  const int* ep = experts.data_ptr<int>();
  const int* rp = row_map.data_ptr<int>();
  float* zp = z.data_ptr<float>();
  if (maxr == 1) tr_gemv_launch<1>(grid, st, K, xp, tp, ep, rp, zp, (int)Kt, (int)Nt, (int)L, mad, scale);
  else if (maxr == 2) tr_gemv_launch<2>(grid, st, K, xp, tp, ep, rp, zp, (int)Kt, (int)Nt, (int)L, mad, scale);
  else if (maxr <= 4) tr_gemv_launch<4>(grid, st, K, xp, tp, ep, rp, zp, (int)Kt, (int)Nt, (int)L, mad, scale);
  else tr_gemv_launch<8>(grid, st, K, xp, tp, ep, rp, zp, (int)Kt, (int)Nt, (int)L, mad, scale);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
