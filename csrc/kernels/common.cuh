// Shared device helpers for the sm_100a kernels of vllm_moet_b200.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#define MOET_DEVICE __device__ __forceinline__

namespace moet {

// Status codes written by kernels into a device int instead of trapping.
enum Status : int {
  kOk = 0,
  kBadIndex = 1,      // an index (slot, expert, position) was out of range
  kTimeout = 2,       // a bounded wait gave up
  kBadSize = 3,
  kBadValue = 4,     // a non-finite value where a finite one is required
};

// Programmatic dependent launch.  Kernels launched with launch_k() may start
// while the previous kernel on the stream is still running; each such kernel
// (1) may touch only immutable data (weights) before pdl_wait(), (2) calls
// pdl_wait() -- which returns once the previous grid has completed and its
// writes are visible -- before any other global read or any global write, and
// (3) calls pdl_trigger() right after, letting the next kernel start its own
// prologue.  Both are no-ops for a kernel launched without the attribute.
MOET_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
MOET_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
MOET_DEVICE void pdl_entry() { pdl_wait(); pdl_trigger(); }
MOET_DEVICE void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

MOET_DEVICE void set_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// UE8M0 byte -> float 2^(b-127).  The byte is exactly the IEEE-754 single
// biased exponent, so b<<23 is the float (b == 0 gives 0, used for 2^-127).
MOET_DEVICE float ue8m0_to_float(uint32_t b) { return __uint_as_float(b << 23); }

MOET_DEVICE uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// D = A(16x32 e4m3, row) * B(32x8 e4m3, col) + C, f32 accumulate.
MOET_DEVICE void mma_e4m3_16832(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1),
        "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

// D = A(16x16 bf16) * B(16x8 bf16) + C
MOET_DEVICE void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

MOET_DEVICE void ldmatrix_x4(uint32_t (&r)[4], const void* smem) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
MOET_DEVICE void ldmatrix_x2(uint32_t (&r)[2], const void* smem) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1]) : "r"(a));
}
MOET_DEVICE void ldmatrix_x4_trans(uint32_t (&r)[4], const void* smem) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
MOET_DEVICE void ldmatrix_x2_trans(uint32_t (&r)[2], const void* smem) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1]) : "r"(a));
}

MOET_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Streaming 128/64-bit global loads that do not allocate in L1.
MOET_DEVICE uint4 ldg_stream_u4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
MOET_DEVICE uint2 ldg_stream_u2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}

MOET_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
MOET_DEVICE float e4m3_to_f32(uint8_t b) {
  __nv_fp8_e4m3 v;
  v.__x = b;
  return static_cast<float>(v);
}

MOET_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Smallest power-of-two exponent e with amax / 2^e <= 448, as a UE8M0 byte.
MOET_DEVICE uint32_t ue8m0_for_amax(float amax) {
  if (!(amax > 0.f)) return 0;  // all-zero group: 2^-127
  // frexp: amax = m * 2^x with m in [0.5, 1); amax/448 <= 2^e
  float r = amax * (1.0f / 448.0f);
  uint32_t bits = __float_as_uint(r);
  int ex = (int)((bits >> 23) & 0xff);         // biased exponent of r
  uint32_t mant = bits & 0x7fffff;
  int e = ex - 127 + (mant != 0 ? 1 : 0);      // ceil(log2(r))
  if (ex == 0) e = -126;                       // subnormal r: tiny amax
  e = max(-127, min(127, e));
  return (uint32_t)(e + 127);
}

MOET_DEVICE uint8_t f32_to_e4m3(float x) {
  __nv_fp8_e4m3 v(x);  // satfinite, round-to-nearest-even
  return *reinterpret_cast<uint8_t*>(&v);
}

// e2m1x2 conversion (hardware cvt, round-to-nearest-even, saturating).
MOET_DEVICE uint32_t f32x8_to_e2m1x8(const float* f) {
  uint32_t val;
  asm volatile(
      "{\n.reg .b8 b0, b1, b2, b3;\n"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n"
      "mov.b32 %0, {b0, b1, b2, b3};\n}"
      : "=r"(val)
      : "f"(f[0]), "f"(f[1]), "f"(f[2]), "f"(f[3]), "f"(f[4]), "f"(f[5]), "f"(f[6]), "f"(f[7]));
  return val;
}

}  // namespace moet

#include <cstdlib>
#include <mutex>
#include <unordered_set>
#include <utility>
// Host: allow a kernel the device's whole opt-in dynamic shared memory, once per
// kernel.  The attribute is per function, not per launch: setting it to each
// launch's own size would leave it at the LAST size, and a CUDA-graph node
// captured earlier with a larger size is then over the limit whenever the node is
// launched on its own.  The attribute is a ceiling only; occupancy follows the
// size each launch requests.
inline void moet_allow_max_smem(const void* kern) {
  static std::mutex mu;
  static std::unordered_set<const void*> done;
  static int optin = 0;
  std::lock_guard<std::mutex> lk(mu);
  if (done.count(kern)) return;
  if (!optin) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  }
  int static_bytes = 0;
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, kern) == cudaSuccess) static_bytes = (int)fa.sharedSizeBytes;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - static_bytes);
  done.insert(kern);
}
template <typename... KArgs>
inline void moet_allow_max_smem(void (*kern)(KArgs...)) {
  moet_allow_max_smem(reinterpret_cast<const void*>(kern));
}
// Host: launch with the programmatic-stream-serialization attribute (PDL) unless
// MOET_PDL=0.  Captured into CUDA graphs as programmatic dependency edges.
inline bool moet_pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("MOET_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
inline void launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                     Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = moet_pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}
