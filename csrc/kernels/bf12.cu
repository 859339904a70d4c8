// bf12 decode: class nibble + LO byte -> bf16, then the escape scatter.
// Layout (see formats/bf12.py): classes[i/2] holds the nibble of weight i
// (even i in the low nibble); hi byte = lut[nibble]; word = hi << 8 | lo[i];
// escaped weights take their hi byte from the escape list.  Each thread
// decodes 8 weights (4 class bytes -> one 32-bit load, 8 LO bytes -> one 64-bit load).
#include "common.cuh"
#include "torch_glue.h"

namespace moet {

__global__ void bf12_decode_kernel(const uint8_t* __restrict__ cls, const uint8_t* __restrict__ lo,
                                   const uint8_t* __restrict__ lut, long long n, uint16_t* __restrict__ out) {
  pdl_entry();
  __shared__ uint8_t L[16];
  if (threadIdx.x < 16) L[threadIdx.x] = lut[threadIdx.x];
  __syncthreads();
  const long long base = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (base >= n) return;
  if (base + 8 <= n) {
    const uint32_t c = *reinterpret_cast<const uint32_t*>(cls + base / 2);
    const uint2 l = *reinterpret_cast<const uint2*>(lo + base);
    const uint32_t lw[2] = {l.x, l.y};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const uint32_t b = (c >> (8 * j)) & 0xFF;
      const uint32_t h0 = L[b & 0xF], h1 = L[b >> 4];
      const uint32_t lo0 = (lw[j >> 1] >> (16 * (j & 1))) & 0xFF, lo1 = (lw[j >> 1] >> (16 * (j & 1) + 8)) & 0xFF;
      o[j] = (h0 << 8 | lo0) | ((h1 << 8 | lo1) << 16);
    }
    *reinterpret_cast<uint4*>(out + base) = make_uint4(o[0], o[1], o[2], o[3]);
  } else {
    for (long long i = base; i < n; i++) {
      const uint32_t b = cls[i / 2];
      const uint32_t nib = (i & 1) ? (b >> 4) : (b & 0xF);
      out[i] = (uint16_t)(L[nib] << 8 | lo[i]);
    }
  }
}

__global__ void bf12_escape_kernel(const long long* __restrict__ pos, const uint8_t* __restrict__ hi, long long m,
                                   const uint8_t* __restrict__ lo, uint16_t* __restrict__ out) {
  pdl_entry();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m) return;
  const long long p = pos[i];
  out[p] = (uint16_t)((uint32_t)hi[i] << 8 | lo[p]);
}

}  // namespace moet

using namespace moet;

void bf12_decode(torch::Tensor cls, torch::Tensor lo, torch::Tensor lut, torch::Tensor esc_pos, torch::Tensor esc_hi,
                 torch::Tensor out) {
  const long long n = lo.numel();
  TORCH_CHECK(out.numel() == n && out.scalar_type() == at::kBFloat16 && out.is_contiguous(), "bf12_decode: out");
  TORCH_CHECK(cls.numel() == (n + 1) / 2 && lut.numel() == 16 && esc_pos.scalar_type() == at::kLong,
              "bf12_decode: plane shapes");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(cls.data_ptr()) % 4 == 0 && reinterpret_cast<uintptr_t>(lo.data_ptr()) % 8 == 0 &&
              reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0, "bf12_decode: alignment");
  if (n == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  const int threads = 256;
  const long long groups = (n + 7) / 8;
  launch_k(bf12_decode_kernel, (unsigned)((groups + threads - 1) / threads), threads, 0, stream,
           (const uint8_t*)cls.data_ptr(), (const uint8_t*)lo.data_ptr(), (const uint8_t*)lut.data_ptr(), n,
           (uint16_t*)out.data_ptr());
  const long long m = esc_pos.numel();
  if (m)
    launch_k(bf12_escape_kernel, (unsigned)((m + threads - 1) / threads), threads, 0, stream,
             (const long long*)esc_pos.data_ptr(), (const uint8_t*)esc_hi.data_ptr(), m, (const uint8_t*)lo.data_ptr(),
             (uint16_t*)out.data_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
