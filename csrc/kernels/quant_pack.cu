// Load-time expert quantisation on the GPU.
//   nvfp4_quant  : float [N,K] -> NVFP4 (packed e2m1 [N,K/2], e4m3 block-16 scales, f32 tensor scale)
//   w2_quant_pack: NVFP4 expert -> 2-bit sign-symmetric codes + UE8M0 block-32 scales,
//                  written straight into the fragment-major code / scale planes
//                  (and optionally the e2m1 nibble plane for the FP4 delta tier).
// The arithmetic is the golden pipeline of vllm_moet_b200.formats.codebook
// (reference P:12256-12397): exact dequant in f64, exponent =
// round(log2(amax/6)) clamped to [-127, 127], snap to the e2m1 grid at the
// midpoints (ties to the lower magnitude), sign from the sign bit; zero-sign
// mode 0 keeps signs, mode 1 alternates by k parity.  Per-tensor counters
// of exact zeros / negative zeros let the host apply the "auto" rule.
#include "common.cuh"
#include "torch_glue.h"

namespace moet {

// one thread per (row, 16-block)
MOET_DEVICE void nvfp4_quant_body(long long idx, const float* __restrict__ w, int N, int K, float ts,
                                  uint8_t* __restrict__ packed, uint8_t* __restrict__ sf) {
  const long long nblk = (long long)N * (K / 16);
  if (idx >= nblk) return;
  const int r = idx / (K / 16), b = idx % (K / 16);
  const float* src = w + (size_t)r * K + b * 16;
  float x[16];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; i++) { x[i] = src[i]; amax = fmaxf(amax, fabsf(x[i])); }
  const float s = fminf(__fdiv_rn(__fdiv_rn(amax, 6.0f), ts), 448.0f);
  const uint8_t sq = f32_to_e4m3(s);
  __nv_fp8_e4m3 sv; *reinterpret_cast<uint8_t*>(&sv) = sq;
  const float scale = float(sv) * ts;
  const float inv = scale > 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
  float q[16];
#pragma unroll
  for (int i = 0; i < 16; i++) q[i] = x[i] * inv;
  uint2 out;
  out.x = f32x8_to_e2m1x8(q);
  out.y = f32x8_to_e2m1x8(q + 8);
  *reinterpret_cast<uint2*>(packed + (size_t)r * (K / 2) + b * 8) = out;
  sf[(size_t)r * (K / 16) + b] = sq;
}

__global__ void nvfp4_quant_kernel(const float* __restrict__ w, int N, int K, float ts,
                                   uint8_t* __restrict__ packed, uint8_t* __restrict__ sf) {
  nvfp4_quant_body((long long)blockIdx.x * blockDim.x + threadIdx.x, w, N, K, ts, packed, sf);
}

// batched over experts (blockIdx.y), per-expert tensor scale ts[e]
__global__ void nvfp4_quant_batched_kernel(const float* __restrict__ w, int N, int K, const double* __restrict__ ts,
                                           uint8_t* __restrict__ packed, uint8_t* __restrict__ sf) {
  const size_t e = blockIdx.y;
  nvfp4_quant_body((long long)blockIdx.x * blockDim.x + threadIdx.x, w + e * N * K, N, K, (float)ts[e],
                   packed + e * N * (K / 2), sf + e * N * (K / 16));
}

__constant__ double kE2M1Val[8] = {0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0};

// one thread per (row, 32-block)
MOET_DEVICE void w2_quant_pack_body(long long idx, const uint8_t* __restrict__ packed, const uint8_t* __restrict__ sf,
                                    double ts, int N, int K, int zero_mode, uint8_t* __restrict__ codes_plane,
                                    uint8_t* __restrict__ scale_plane, uint8_t* __restrict__ fp4_plane,
                                    unsigned long long* __restrict__ counters) {
  const int KS = K / 32, KC = K / 64;
  if (idx >= (long long)N * KS) return;
  const int r = idx / KS, ks = idx % KS;
  double v[32];
  double amax = 0.0;
#pragma unroll
  for (int i = 0; i < 32; i++) {
    const int k = ks * 32 + i;
    const uint8_t byte = packed[(size_t)r * (K / 2) + k / 2];
    const uint8_t nib = (k & 1) ? (byte >> 4) : (byte & 0xF);
    __nv_fp8_e4m3 s8; *reinterpret_cast<uint8_t*>(&s8) = sf[(size_t)r * (K / 16) + k / 16];
    double val = kE2M1Val[nib & 7] * (double)float(s8) * ts;
    if (nib & 8) val = -val;
    v[i] = val;
    amax = fmax(amax, fabs(val));
  }
  double e = -127.0;
  if (amax > 0.0) e = fmin(127.0, fmax(-127.0, rint(log2(amax / 6.0 + 1e-30))));
  // rint is ties-to-even; torch.round is ties-to-even too.
  const uint8_t sbyte = (uint8_t)(e + 127.0);
  const double inv = exp2(-e);
  const int nb = r >> 4, rr = r & 15, tile = rr >> 3, g = rr & 7;
  const int kb = ks >> 1, k32 = ks & 1;
  unsigned long long nzero = 0, nneg = 0;
  uint8_t nibs[32];
#pragma unroll
  for (int i = 0; i < 32; i++) {
    const double u = v[i] * inv;
    const double a = fabs(u);
    // bucketize on midpoints [0.25,0.75,1.25,1.75,2.5,3.5,5.0], right=False (a == mid -> lower)
    int mag = (a > 0.25) + (a > 0.75) + (a > 1.25) + (a > 1.75) + (a > 2.5) + (a > 3.5) + (a > 5.0);
    bool neg = signbit(u);
    if (u == 0.0) {
      nzero++; nneg += neg ? 1 : 0;
      if (zero_mode == 1) neg = ((ks * 32 + i) & 1) != 0;
    }
    nibs[i] = (uint8_t)(mag | (neg ? 8 : 0));
  }
  // codes: nibble -> {0:-4,1:-1,2:+1,3:+4}
  uint8_t codes[32];
#pragma unroll
  for (int i = 0; i < 32; i++) {
    const int mag = nibs[i] & 7; const bool neg = nibs[i] & 8;
    codes[i] = neg ? (mag >= 5 ? 0 : 1) : (mag >= 5 ? 3 : 2);
  }
  // plane byte for (nb, kb, g, t, tile, k32, half): ((((nb*KC+kb)*8+g)*4+t)*8 + tile*4 + k32*2 + half
#pragma unroll
  for (int half = 0; half < 2; half++)
#pragma unroll
    for (int t = 0; t < 4; t++) {
      const int i0 = half * 16 + t * 4;
      const uint8_t byte = codes[i0] | (codes[i0 + 1] << 2) | (codes[i0 + 2] << 4) | (codes[i0 + 3] << 6);
      const size_t lane_base = ((((size_t)nb * KC + kb) * 8 + g) * 4 + t);
      codes_plane[lane_base * 8 + tile * 4 + k32 * 2 + half] = byte;
      if (fp4_plane) {
        const uint8_t b0 = nibs[i0] | (nibs[i0 + 1] << 4), b1 = nibs[i0 + 2] | (nibs[i0 + 3] << 4);
        uint8_t* d = fp4_plane + lane_base * 16 + (tile * 4 + k32 * 2 + half) * 2;
        d[0] = b0; d[1] = b1;
      }
    }
  scale_plane[((size_t)nb * KS + ks) * 16 + rr] = sbyte;
  if (counters && nzero) { atomicAdd(&counters[0], nzero); atomicAdd(&counters[1], nneg); }
}

__global__ void w2_quant_pack_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ sf, double ts,
                                     int N, int K, int zero_mode, uint8_t* __restrict__ codes_plane,
                                     uint8_t* __restrict__ scale_plane, uint8_t* __restrict__ fp4_plane,
                                     unsigned long long* __restrict__ counters) {
  w2_quant_pack_body((long long)blockIdx.x * blockDim.x + threadIdx.x, packed, sf, ts, N, K, zero_mode, codes_plane,
                     scale_plane, fp4_plane, counters);
}

// Batched over experts (blockIdx.y) into slot rows of a pool.  zero_mode 0 / 1 as above and
// counting zeros per expert; zero_mode 2 is the second pass of the "auto" rule: an expert whose
// counters show a sign-unbalanced set of exact zeros (the minority sign under 5 %) is packed
// again with mode 1, every other expert is left as it is -- no host round trip.
__global__ void w2_quant_pack_batched_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ sf,
                                             const double* __restrict__ ts, int N, int K, int zero_mode,
                                             uint8_t* __restrict__ pool, long long slot_stride, long long off_c,
                                             long long off_s, unsigned long long* __restrict__ counters) {
  const size_t e = blockIdx.y;
  unsigned long long* cnt = counters + 2 * e;
  int mode = zero_mode;
  if (zero_mode == 2) {
    const unsigned long long nz = cnt[0], nneg = cnt[1];
    if (!(nz && (double)min(nneg, nz - nneg) < 0.05 * (double)nz)) return;
    mode = 1;
  }
  uint8_t* slot = pool + e * slot_stride;
  w2_quant_pack_body((long long)blockIdx.x * blockDim.x + threadIdx.x, packed + e * N * (K / 2),
                     sf + e * N * (K / 16), ts[e], N, K, mode, slot + off_c, slot + off_s, nullptr,
                     zero_mode == 2 ? nullptr : cnt);
}

}  // namespace moet

using namespace moet;

void nvfp4_quant(torch::Tensor w, double ts, torch::Tensor packed, torch::Tensor sf) {
  const int N = w.size(0), K = w.size(1);
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && K % 16 == 0, "nvfp4_quant: f32 [N, K%16]");
  const long long n = (long long)N * (K / 16);
  if (n == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  nvfp4_quant_kernel<<<(n + 255) / 256, 256, 0, stream>>>(w.data_ptr<float>(), N, K, (float)ts,
                                                          (uint8_t*)packed.data_ptr(), (uint8_t*)sf.data_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void w2_quant_pack(torch::Tensor packed, torch::Tensor sf, double ts, int64_t zero_mode, torch::Tensor codes_plane,
                   torch::Tensor scale_plane, c10::optional<torch::Tensor> fp4_plane,
                   c10::optional<torch::Tensor> counters) {
  const int N = packed.size(0), K = packed.size(1) * 2;
  TORCH_CHECK(N % 16 == 0 && K % 64 == 0, "w2_quant_pack: N % 16, K % 64");
  TORCH_CHECK(codes_plane.numel() >= (long long)N * K / 4 && scale_plane.numel() >= (long long)N * K / 32,
              "w2_quant_pack: plane sizes");
  const long long n = (long long)N * (K / 32);
  auto stream = at::cuda::getCurrentCUDAStream();
  w2_quant_pack_kernel<<<(n + 127) / 128, 128, 0, stream>>>(
      (const uint8_t*)packed.data_ptr(), (const uint8_t*)sf.data_ptr(), ts, N, K, (int)zero_mode,
      (uint8_t*)codes_plane.data_ptr(), (uint8_t*)scale_plane.data_ptr(), (uint8_t*)opt_ptr(fp4_plane),
      (unsigned long long*)opt_ptr(counters));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// All experts of a chunk in three launches: w [n, N, K] f32 (cuda), ts [n] f64 (the
// per-expert tensor scales), scratch packed [n, N, K/2] / sf [n, N, K/16] u8, counters
// [n, 2] u64 zeroed, slot rows pool [n, slot_stride] (codes at off_c, scales at off_s).
void experts_quant_pack(torch::Tensor w, torch::Tensor ts, torch::Tensor packed, torch::Tensor sf,
                        torch::Tensor counters, torch::Tensor pool, int64_t off_c, int64_t off_s, int64_t zero_mode) {
  const int n = w.size(0), N = w.size(1), K = w.size(2);
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && K % 64 == 0 && N % 16 == 0,
              "experts_quant_pack: w f32 [n, N, K], N % 16, K % 64");
  TORCH_CHECK(ts.scalar_type() == at::kDouble && ts.numel() == n && counters.numel() >= 2 * n &&
              packed.numel() >= (int64_t)n * N * K / 2 && sf.numel() >= (int64_t)n * N * K / 16 &&
              pool.dim() == 2 && pool.size(0) >= n, "experts_quant_pack: shapes");
  if (n == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  const long long nq = (long long)N * (K / 16), np = (long long)N * (K / 32);
  nvfp4_quant_batched_kernel<<<dim3((nq + 255) / 256, n), 256, 0, stream>>>(
      w.data_ptr<float>(), N, K, ts.data_ptr<double>(), (uint8_t*)packed.data_ptr(), (uint8_t*)sf.data_ptr());
  const int first = zero_mode == 1 ? 1 : 0;
  w2_quant_pack_batched_kernel<<<dim3((np + 127) / 128, n), 128, 0, stream>>>(
      (const uint8_t*)packed.data_ptr(), (const uint8_t*)sf.data_ptr(), ts.data_ptr<double>(), N, K, first,
      (uint8_t*)pool.data_ptr(), pool.stride(0), off_c, off_s, (unsigned long long*)counters.data_ptr());
  if (zero_mode == 2)    // "auto"
    w2_quant_pack_batched_kernel<<<dim3((np + 127) / 128, n), 128, 0, stream>>>(
        (const uint8_t*)packed.data_ptr(), (const uint8_t*)sf.data_ptr(), ts.data_ptr<double>(), N, K, 2,
        (uint8_t*)pool.data_ptr(), pool.stride(0), off_c, off_s, (unsigned long long*)counters.data_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
