// RMSNorm (+ residual add) fused with FP8 e4m3 activation quantisation, and
// SwiGLU (+ clamp) fused with the same quantisation.
//
// Activation quantisation: groups of 64 along K, one UE8M0 exponent per
// (row, group) = smallest e with amax/2^e <= 448.  Two byte layouts:
//   layout 0 (natural):  k at position k                 (dense FP8 GEMV/GEMM)
//   layout 1 (w2):       inside each 32-block position 8t+q holds
//                        k = [4t,4t+2,16+4t,18+4t,4t+1,4t+3,17+4t,19+4t][q]
//                        (the A-fragment byte order of the 2-bit expert decode)
// The reference quantises activations in a separate op with 128-wide groups
// (P:4388-4401); here it is fused into the producer and the group is 64 so
// it also matches every K-shard of the experts under TP.
#include "common.cuh"
#include "symm.cuh"
#include "torch_glue.h"

namespace moet {

MOET_DEVICE int w2_pos(int k) {
  int blk = k & ~31, r = k & 31;
  int half = r >> 4, rr = r & 15, t = rr >> 2, jj = rr & 3;
  return blk + 8 * t + (jj & 1) * 4 + half * 2 + (jj >> 1);
}

// Each thread owns VEC consecutive elements; 64/VEC threads share a group.
template <int VEC>
MOET_DEVICE void quant_store(const float (&v)[VEC], int row, int k0, int K, int layout,
                             uint8_t* __restrict__ q, uint8_t* __restrict__ s, int ostride = 0) {
  if (ostride == 0) ostride = K;
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < VEC; i++) amax = fmaxf(amax, fabsf(v[i]));
  constexpr int TPG = 64 / VEC;  // threads per group (consecutive lanes)
  const unsigned mask = __activemask();  // groups are aligned: fully active or fully idle
  for (int o = 1; o < TPG; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(mask, amax, o));
  uint32_t e = ue8m0_for_amax(amax);
  // 1 / 2^(e-127) = 2^(127-e), exact for e in [1, 253]; e == 0 is an all-zero group.
  const float inv = (e >= 1 && e <= 253) ? __uint_as_float((254u - e) << 23) : 0.f;
  uint8_t* qr = q + (size_t)row * ostride;
  if (layout == 0) {
    uint8_t b[VEC];
#pragma unroll
    for (int i = 0; i < VEC; i++) b[i] = f32_to_e4m3(v[i] * inv);
    if constexpr (VEC == 16) {
      *reinterpret_cast<uint4*>(qr + k0) = *reinterpret_cast<uint4*>(b);
    } else if constexpr (VEC == 8) {
      *reinterpret_cast<uint2*>(qr + k0) = *reinterpret_cast<uint2*>(b);
    } else {
#pragma unroll
      for (int i = 0; i < VEC; i++) qr[k0 + i] = b[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < VEC; i++) qr[w2_pos(k0 + i)] = f32_to_e4m3(v[i] * inv);
  }
  if ((threadIdx.x % TPG) == 0) s[(size_t)row * (ostride / 64) + k0 / 64] = (uint8_t)e;
}

// grid = rows, block = H/16 threads (H % 1024 == 0 -> <=... any H multiple of 64 with H/16 <= 1024)
// x_in: [rows, H] bf16; add (optional): [rows, H] bf16, x_out (optional) = x_in + add.
template <int VEC>
__global__ void rmsnorm_quant_kernel(const __nv_bfloat16* __restrict__ x_in,
                                     const __nv_bfloat16* __restrict__ add,
                                     __nv_bfloat16* __restrict__ x_out,
                                     const __nv_bfloat16* __restrict__ w, float eps, int H,
                                     __nv_bfloat16* __restrict__ y_out,
                                     uint8_t* __restrict__ q0, uint8_t* __restrict__ s0,
                                     uint8_t* __restrict__ q1, uint8_t* __restrict__ s1,
                                     int in_stride, int ostride, int ar_on, ArDesc ar) {
  pdl_entry();
  const int row = blockIdx.x;
  const int k0 = threadIdx.x * VEC;
  float v[VEC];
  const __nv_bfloat16* xr = x_in + (size_t)row * in_stride + k0;
#pragma unroll
  for (int i = 0; i < VEC; i++) v[i] = __bfloat162float(xr[i]);
  if (ar_on) {   // all-reduce consumer: x = residual + sum over ranks (rank order) of the pushed partials
    const unsigned long long epoch = ar_epoch(ar);
    if (ar_consumer_wait(ar, epoch)) {
      float s[VEC];
#pragma unroll
      for (int i = 0; i < VEC; i++) s[i] = 0.f;
      for (int r = 0; r < ar.world; r++) {
        const float* src = ar_slot(ar, ar.rank, epoch, r) + (size_t)row * H + k0;
#pragma unroll
        for (int i = 0; i < VEC; i += 4) {
          const float4 f = *reinterpret_cast<const float4*>(src + i);
          s[i] += f.x; s[i + 1] += f.y; s[i + 2] += f.z; s[i + 3] += f.w;
        }
      }
#pragma unroll
      for (int i = 0; i < VEC; i++) v[i] += s[i];
    }
  }
  if (add) {
    const __nv_bfloat16* ar = add + (size_t)row * H + k0;
#pragma unroll
    for (int i = 0; i < VEC; i++) v[i] += __bfloat162float(ar[i]);
  }
  if (x_out) {
#pragma unroll
    for (int i = 0; i < VEC; i++) {
      __nv_bfloat16 b = __float2bfloat16(v[i]);
      x_out[(size_t)row * H + k0 + i] = b;
      v[i] = __bfloat162float(b);  // the residual stream is bf16: normalise what was stored
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VEC; i++) ss += v[i] * v[i];
  ss = warp_sum(ss);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float rinv = rsqrtf(red[0] / (float)H + eps);
#pragma unroll
  for (int i = 0; i < VEC; i++) {
    // round through bf16 like the module output would be
    v[i] = __bfloat162float(__float2bfloat16(v[i] * rinv * __bfloat162float(w[k0 + i])));
  }
  if (y_out) {
#pragma unroll
    for (int i = 0; i < VEC; i++) y_out[(size_t)row * ostride + k0 + i] = __float2bfloat16(v[i]);
  }
  if (q0) quant_store<VEC>(v, row, k0, H, 0, q0, s0, ostride);
  if (q1) quant_store<VEC>(v, row, k0, H, 1, q1, s1, ostride);
  if (ar_on) ar_consumer_done(ar);
}

// SwiGLU: in [rows, 2I] f32 (gate | up), out e4m3 [rows, I].
// act = silu(min(g, L)) * clamp(u, -L, L)   (L <= 0 disables the clamp);
// the product is rounded to bf16 before quantisation (matches a bf16 module).
__global__ void swiglu_quant_kernel(const float* __restrict__ in, int I, float limit,
                                    const int* __restrict__ n_rows, int layout,
                                    uint8_t* __restrict__ q, uint8_t* __restrict__ s,
                                    int nsplit, long long split_stride) {
  pdl_entry();
  const int row = blockIdx.x;
  if (n_rows && row >= *n_rows) return;
  constexpr int VEC = 8;
  for (int k0 = threadIdx.x * VEC; k0 < I; k0 += blockDim.x * VEC) {
    float v[VEC];
    const float* g = in + (size_t)row * 2 * I + k0;
    const float* u = g + I;
#pragma unroll
    for (int i = 0; i < VEC; i++) {
      float gv = g[i], uv = u[i];
      for (int q = 1; q < nsplit; q++) {   // K-slice partials of the expert GEMV, slice order
        gv += g[q * split_stride + i];
        uv += u[q * split_stride + i];
      }
      if (limit > 0.f) { gv = fminf(gv, limit); uv = fminf(fmaxf(uv, -limit), limit); }
      float a = gv / (1.f + __expf(-gv)) * uv;
      v[i] = __bfloat162float(__float2bfloat16(a));
    }
    quant_store<VEC>(v, row, k0, I, layout, q, s);
  }
}

// Plain quantisation of a bf16 / f32 matrix.
template <typename T>
__global__ void quant_kernel(const T* __restrict__ x, int K, int in_stride, int layout,
                             uint8_t* __restrict__ q, uint8_t* __restrict__ s) {
  pdl_entry();
  const int row = blockIdx.x;
  constexpr int VEC = 8;
  for (int k0 = threadIdx.x * VEC; k0 < K; k0 += blockDim.x * VEC) {
    float v[VEC];
#pragma unroll
    for (int i = 0; i < VEC; i++) v[i] = (float)x[(size_t)row * in_stride + k0 + i];
    quant_store<VEC>(v, row, k0, K, layout, q, s);
  }
}

}  // namespace moet

using namespace moet;


void rmsnorm_quant(torch::Tensor x, c10::optional<torch::Tensor> add, c10::optional<torch::Tensor> x_out,
                   torch::Tensor w, double eps, c10::optional<torch::Tensor> y_out,
                   c10::optional<torch::Tensor> q0, c10::optional<torch::Tensor> s0,
                   c10::optional<torch::Tensor> q1, c10::optional<torch::Tensor> s1, int64_t ostride,
                   c10::optional<torch::Tensor> ar) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16, "x must be cuda bf16");
  const int rows = x.size(0), H = w.size(0);
  TORCH_CHECK(x.stride(1) == 1, "x inner stride must be 1");
  TORCH_CHECK(H % 64 == 0, "H must be a multiple of 64");
  if (rows == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  TORCH_CHECK(H <= 16384, "H too large for rmsnorm_quant (max 16384)");
  const int vec = H >= 512 ? 16 : (H >= 256 ? 8 : 4);
  TORCH_CHECK(H >= 128, "rmsnorm_quant: H must be >= 128");
  const int threads = H / vec;
  auto kern = vec == 16 ? rmsnorm_quant_kernel<16> : (vec == 8 ? rmsnorm_quant_kernel<8> : rmsnorm_quant_kernel<4>);
  const int ar_on = ar.has_value() && ar->defined();
  ArDesc d{};
  if (ar_on) {
    d = ar_desc_from(*ar);
    TORCH_CHECK(x_out.has_value() && x_out->defined() && !(add.has_value() && add->defined()),
                "rmsnorm_quant: the all-reduce consumer writes x_out = x + sum of partials (no add)");
    TORCH_CHECK((int64_t)rows * H <= d.cap, "rmsnorm_quant: rows*H exceeds the all-reduce slot");
  }
  launch_k(kern, rows, threads, 0, stream, 
      (const __nv_bfloat16*)x.data_ptr(), (const __nv_bfloat16*)opt_ptr(add),
      (__nv_bfloat16*)opt_ptr(x_out), (const __nv_bfloat16*)w.data_ptr(), (float)eps, H,
      (__nv_bfloat16*)opt_ptr(y_out), (uint8_t*)opt_ptr(q0), (uint8_t*)opt_ptr(s0),
      (uint8_t*)opt_ptr(q1), (uint8_t*)opt_ptr(s1), (int)x.stride(0), (int)(ostride ? ostride : H), ar_on, d);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void swiglu_quant(torch::Tensor in, double limit, c10::optional<torch::Tensor> n_rows, int64_t layout,
                  torch::Tensor q, torch::Tensor s) {
  // in: [rows, 2I] or [nsplit, rows, 2I] (K-slice partials, summed in slice order)
  TORCH_CHECK(in.scalar_type() == at::kFloat && in.is_contiguous(), "in must be contiguous f32");
  const int nsplit = in.dim() == 3 ? in.size(0) : 1;
  const long long split_stride = in.dim() == 3 ? in.stride(0) : 0;
  const int rows = in.size(-2), I = in.size(-1) / 2;
  TORCH_CHECK(I % 64 == 0, "I must be a multiple of 64");
  if (rows == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  int threads = std::min(256, I / 8);
  launch_k(swiglu_quant_kernel, rows, threads, 0, stream, in.data_ptr<float>(), I, (float)limit,
                                                    (const int*)opt_ptr(n_rows), (int)layout,
                                                    (uint8_t*)q.data_ptr(), (uint8_t*)s.data_ptr(),
                                                    nsplit, split_stride);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void quant_fp8(torch::Tensor x, int64_t layout, torch::Tensor q, torch::Tensor s) {
  const int rows = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 64 == 0 && x.stride(1) == 1, "K must be a multiple of 64, inner stride 1");
  if (rows == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  int threads = std::min(256, K / 8);
  if (x.scalar_type() == at::kBFloat16)
    launch_k(quant_kernel<__nv_bfloat16>, rows, threads, 0, stream, (const __nv_bfloat16*)x.data_ptr(), K,
                                                             (int)x.stride(0), (int)layout,
                                                             (uint8_t*)q.data_ptr(), (uint8_t*)s.data_ptr());
  else if (x.scalar_type() == at::kFloat)
    launch_k(quant_kernel<float>, rows, threads, 0, stream, x.data_ptr<float>(), K, (int)x.stride(0), (int)layout,
                                                     (uint8_t*)q.data_ptr(), (uint8_t*)s.data_ptr());
  else
    TORCH_CHECK(false, "quant_fp8: bf16 or f32 input");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
