// Persistent, TMA-fed FP8 GEMV for decode: out[T, N] = A[T, K] * W[N, K]^T,
// W e4m3 row-major with UE8M0 128x128 block scales, A e4m3 with UE8M0 per-64
// scales, T <= 8 tokens.
//
// The weight-streaming GEMV in gemv_fp8.cu issues one batch of loads per CTA
// and retires; at 3 tokens it reaches ~2 TB/s, latency-bound by CTA waves.
// Here each SM runs one persistent CTA that streams 16-row weight blocks
// through a ring of shared-memory stages filled by cp.async.bulk (one copy
// per row, rows padded by 16 bytes so ldmatrix is conflict-free) completing
// on mbarriers, kRing stages in flight, so HBM sees a continuous stream.
// Eight warps split each block's K range; each takes m16n8k32 e4m3 MMAs with
// the weight rows as A (ldmatrix.x4) and the tokens as B (ldmatrix.x2 from
// the activation rows staged once in shared memory), applies the weight and
// activation scales per 64-k chunk, and the warps' partial sums are reduced
// through shared memory before the next block.  All waits are bounded.
#include "common.cuh"
#include "symm.cuh"
#include "torch_glue.h"

namespace moet {

namespace gs {
constexpr int kRows = 16;        // rows per stage
constexpr int kWarps = 8;
constexpr int kMaxRing = 4;      // stages in flight (as many as fit in shared memory, >= 2)
constexpr int kMaxK = 8192;
constexpr int kMaxT = 8;

MOET_DEVICE uint32_t s32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
MOET_DEVICE void bar_init(uint64_t* b, int n) { asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(s32(b)), "r"(n)); }
MOET_DEVICE void bar_expect(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s32(b)), "r"(bytes));
}
MOET_DEVICE bool bar_try(uint64_t* b, uint32_t par) {
  uint32_t ok;
  asm volatile("{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
               : "=r"(ok) : "r"(s32(b)), "r"(par) : "memory");
  return ok != 0;
}
MOET_DEVICE bool bar_wait(uint64_t* b, uint32_t par) {
  for (uint32_t i = 0; i < (1u << 22); i++)
    if (bar_try(b, par)) return true;
  return false;
}
MOET_DEVICE void bulk(void* dst, const void* src, uint32_t bytes, uint64_t* b) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(s32(dst)), "l"(src), "r"(bytes), "r"(s32(b)) : "memory");
}
}  // namespace gs

struct GemvStreamArgs {
  const uint8_t* A; const uint8_t* sA; long long a_stride, sa_stride;
  const uint8_t* W; const uint8_t* sW; int sw_cols;
  void* out; long long out_stride; int out_f32;
  const __nv_bfloat16* resid;
  int T, N, K;
  int ring;
  int* status;
  // optional fused RMSNorm + e4m3 quantisation of a bf16 input (replaces A / sA)
  const __nv_bfloat16* xin; long long xin_stride; const __nv_bfloat16* gamma; float eps;
  // optional residual add before the norm: x = bf16(xin + xadd), written to xout by CTA 0
  const __nv_bfloat16* xadd; __nv_bfloat16* xout; long long xadd_stride;
  // fused TP all-reduce: push the output instead of storing it / consume into the norm input
  int ar_push, ar_consume;
  ArDesc ar;
};

// 8 bf16 of row r at column c of (xin [+ xadd | + all-reduced partials]), the sum rounded to
// bf16 as the residual stream stores it
MOET_DEVICE void gs_load8(const GemvStreamArgs& p, int r, int c, float (&v)[8], unsigned long long epoch) {
  const uint4 a = *reinterpret_cast<const uint4*>(p.xin + (size_t)r * p.xin_stride + c);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&a);
  if (p.ar_consume) {
    float s[8];
#pragma unroll
    for (int q = 0; q < 8; q++) s[q] = 0.f;
    for (int w = 0; w < p.ar.world; w++) {
      const float4* src = reinterpret_cast<const float4*>(ar_slot(p.ar, p.ar.rank, epoch, w) + (size_t)r * p.K + c);
      const float4 f0 = src[0], f1 = src[1];
      s[0] += f0.x; s[1] += f0.y; s[2] += f0.z; s[3] += f0.w;
      s[4] += f1.x; s[5] += f1.y; s[6] += f1.z; s[7] += f1.w;
    }
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const float2 f = __bfloat1622float2(h[q]);
      v[2 * q] = __bfloat162float(__float2bfloat16(f.x + s[2 * q]));
      v[2 * q + 1] = __bfloat162float(__float2bfloat16(f.y + s[2 * q + 1]));
    }
  } else if (p.xadd) {
    const uint4 b = *reinterpret_cast<const uint4*>(p.xadd + (size_t)r * p.xadd_stride + c);
    const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const float2 f = __bfloat1622float2(h[q]), g = __bfloat1622float2(hb[q]);
      v[2 * q] = __bfloat162float(__float2bfloat16(f.x + g.x));
      v[2 * q + 1] = __bfloat162float(__float2bfloat16(f.y + g.y));
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; q++) { const float2 f = __bfloat1622float2(h[q]); v[2 * q] = f.x; v[2 * q + 1] = f.y; }
  }
}

__global__ void __launch_bounds__(gs::kWarps * 32, 1) gemv_stream_kernel(GemvStreamArgs p) {
  using namespace gs;
  extern __shared__ __align__(128) uint8_t sm[];
  const int KP = p.K + 16;                                  // padded row stride (bytes)
  const int kRing = p.ring;
  uint8_t* ring = sm;                                       // kRing x [16][KP]
  uint8_t* xs = ring + (size_t)kRing * kRows * KP;          // [8][KP] activations
  float* red = reinterpret_cast<float*>(xs + (size_t)kMaxT * KP);   // [warps][16][8]
  float* sas = red + 2 * kWarps * kRows * kMaxT;            // [8][K/64] activation scales (as floats)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sas + kMaxT * (kMaxK / 64));   // red: 2 buffers
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int nblocks = (p.N + kRows - 1) / kRows;
  const int first = blockIdx.x, step = gridDim.x;
  const int nmine = first < nblocks ? (nblocks - first + step - 1) / step : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRing; s++) bar_init(&bars[s], 1);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();
  auto issue = [&](int i) {      // i-th block of this CTA -> stage i % kRing
    const int rb = first + i * step, s = i % kRing;
    const int r0 = rb * kRows, nr = min(kRows, p.N - r0);
    bar_expect(&bars[s], (uint32_t)(nr * p.K));
    for (int r = 0; r < nr; r++)
      bulk(ring + ((size_t)s * kRows + r) * KP, p.W + (size_t)(r0 + r) * p.K, (uint32_t)p.K, &bars[s]);
  };
  // weights are immutable: start the stream before waiting on the previous kernel
  if (threadIdx.x == 0)
    for (int i = 0; i < min(kRing, nmine); i++) issue(i);
  pdl_entry();
  const int ng = p.K / 64;
  const unsigned long long epoch = (p.ar_push || p.ar_consume) ? ar_epoch(p.ar) : 0ull;
  if (p.ar_consume && !ar_consumer_wait(p.ar, epoch)) {
    ar_consumer_done(p.ar);
    // timed out (status records kTimeout): drain the weight copies already in flight, then leave
    if (threadIdx.x == 0)
      for (int i = 0; i < min(kRing, nmine); i++) bar_wait(&bars[i], 0u);
    __syncthreads();
    return;
  }
  if (p.xin == nullptr) {
    // activations (zero rows beyond T) -> shared memory
    for (int i = threadIdx.x; i < kMaxT * (p.K / 16); i += blockDim.x) {
      const int r = i / (p.K / 16), c = (i % (p.K / 16)) * 16;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r < p.T) v = *reinterpret_cast<const uint4*>(p.A + (size_t)r * p.a_stride + c);
      *reinterpret_cast<uint4*>(xs + (size_t)r * KP + c) = v;
    }
    for (int i = threadIdx.x; i < kMaxT * ng; i += blockDim.x) {
      const int r = i / ng, c = i % ng;
      sas[i] = r < p.T ? ue8m0_to_float(p.sA[(size_t)r * p.sa_stride + c]) : 0.f;
    }
  } else {
    // fused RMSNorm + quantisation (rounding as rmsnorm_quant: bf16 module output, then
    // e4m3 with a UE8M0 scale per 64), compact so the code a CTA fetches once stays small:
    // pass 1 -- per-row sums of squares, one 8-element vector per thread and step;
    // pass 2 -- 8 consecutive lanes per 64-group: normalise, group amax by shuffles,
    // scale and convert their 8 elements each.
    float* ssq = red;                                        // [kMaxT] row sums of squares
    if (threadIdx.x < kMaxT) ssq[threadIdx.x] = 0.f;
    __syncthreads();
    const int vpr = p.K / 8;                                 // 8-element vectors per row
#pragma unroll 1
    for (int r = 0; r < p.T; r++) {
      float acc = 0.f;
      for (int i = threadIdx.x; i < vpr; i += blockDim.x) {
        float v[8];
        gs_load8(p, r, i * 8, v, epoch);
#pragma unroll
        for (int q = 0; q < 8; q++) acc = fmaf(v[q], v[q], acc);
      }
      acc = warp_sum(acc);
      if (lane == 0) atomicAdd(&ssq[r], acc);
    }
    __syncthreads();
    const int units = p.T * vpr, padded = (units + blockDim.x - 1) / blockDim.x * blockDim.x;
#pragma unroll 1
    for (int u = threadIdx.x; u < padded; u += blockDim.x) {
      const bool live = u < units;
      const int r = live ? u / vpr : 0, e8 = live ? u - r * vpr : 0;
      float y[8];
      float amax = 0.f;
      if (live) {
        gs_load8(p, r, e8 * 8, y, epoch);
        if (p.xout && blockIdx.x == 0) {       // the summed residual stream, written once
          uint32_t o[4];
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const __nv_bfloat162 b2 = __floats2bfloat162_rn(y[2 * q], y[2 * q + 1]);
            o[q] = *reinterpret_cast<const uint32_t*>(&b2);
          }
          *reinterpret_cast<uint4*>(p.xout + (size_t)r * p.K + e8 * 8) = make_uint4(o[0], o[1], o[2], o[3]);
        }
        const float rinv = rsqrtf(ssq[r] / (float)p.K + p.eps);
        const uint4 gv = reinterpret_cast<const uint4*>(p.gamma)[e8];
        const __nv_bfloat162* gg = reinterpret_cast<const __nv_bfloat162*>(&gv);
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const float2 g2 = __bfloat1622float2(gg[q]);
          y[2 * q] = __bfloat162float(__float2bfloat16(y[2 * q] * rinv * g2.x));
          y[2 * q + 1] = __bfloat162float(__float2bfloat16(y[2 * q + 1] * rinv * g2.y));
          amax = fmaxf(amax, fmaxf(fabsf(y[2 * q]), fabsf(y[2 * q + 1])));
        }
      }
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
      if (live) {
        const uint32_t e = ue8m0_for_amax(amax);
        const float inv = (e >= 1 && e <= 253) ? __uint_as_float((254u - e) << 23) : 0.f;
        uint32_t w[2];
#pragma unroll
        for (int h = 0; h < 2; h++)
          w[h] = (uint32_t)f32_to_e4m3(y[4 * h] * inv) | ((uint32_t)f32_to_e4m3(y[4 * h + 1] * inv) << 8) |
                 ((uint32_t)f32_to_e4m3(y[4 * h + 2] * inv) << 16) | ((uint32_t)f32_to_e4m3(y[4 * h + 3] * inv) << 24);
        *reinterpret_cast<uint2*>(xs + (size_t)r * KP + e8 * 8) = make_uint2(w[0], w[1]);
        if ((e8 & 7) == 0) sas[r * ng + (e8 >> 3)] = ue8m0_to_float(e);
      }
    }
    // rows beyond T: zero activations and scales
    for (int i = threadIdx.x; i < (kMaxT - p.T) * (p.K / 16); i += blockDim.x) {
      const int r = p.T + i / (p.K / 16), c = (i % (p.K / 16)) * 16;
      *reinterpret_cast<uint4*>(xs + (size_t)r * KP + c) = make_uint4(0, 0, 0, 0);
    }
    for (int i = p.T * ng + threadIdx.x; i < kMaxT * ng; i += blockDim.x) sas[i] = 0.f;
  }
  __syncthreads();
  if (p.ar_consume) ar_consumer_done(p.ar);   // the receive slots are no longer read
  const int nchunks = p.K / 64;
  const int cpw = (nchunks + kWarps - 1) / kWarps;          // 64-k chunks per warp
  const int c_lo = warp * cpw, c_hi = min(nchunks, c_lo + cpw);
  for (int i = 0; i < nmine; i++) {
    const int s = i % kRing;
    const int rb = first + i * step, r0 = rb * kRows;
    const uint8_t* swr = p.sW + (size_t)(r0 >> 7) * p.sw_cols;
    const bool ok = bar_wait(&bars[s], (uint32_t)((i / kRing) & 1));
    if (!__syncthreads_and(ok)) {
      if (threadIdx.x == 0) set_status(p.status, kTimeout);
      return;
    }
    const uint8_t* wst = ring + (size_t)s * kRows * KP;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c = c_lo; c < c_hi; c++) {
      float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t a[4], b[2];
      ldmatrix_x4(a, wst + (size_t)(lane & 15) * KP + c * 64 + (lane >> 4) * 16);
      ldmatrix_x2(b, xs + (size_t)(lane & 7) * KP + c * 64 + ((lane >> 3) & 1) * 16);
      mma_e4m3_16832(d0, a, b[0], b[1], d0);
      ldmatrix_x4(a, wst + (size_t)(lane & 15) * KP + c * 64 + 32 + (lane >> 4) * 16);
      ldmatrix_x2(b, xs + (size_t)(lane & 7) * KP + c * 64 + 32 + ((lane >> 3) & 1) * 16);
      mma_e4m3_16832(d1, a, b[0], b[1], d1);
      const float ws = ue8m0_to_float(swr[c >> 1]);
      const float s0 = ws * sas[(2 * t) * ng + c];
      const float s1 = ws * sas[(2 * t + 1) * ng + c];
      acc[0] = fmaf(d0[0] + d1[0], s0, acc[0]);
      acc[1] = fmaf(d0[1] + d1[1], s1, acc[1]);
      acc[2] = fmaf(d0[2] + d1[2], s0, acc[2]);
      acc[3] = fmaf(d0[3] + d1[3], s1, acc[3]);
    }
    // partial sums -> red[i & 1]; one barrier frees stage s and publishes red
    float* rw = red + ((size_t)(i & 1) * kWarps + warp) * kRows * kMaxT;
    rw[g * kMaxT + 2 * t] = acc[0];
    rw[g * kMaxT + 2 * t + 1] = acc[1];
    rw[(g + 8) * kMaxT + 2 * t] = acc[2];
    rw[(g + 8) * kMaxT + 2 * t + 1] = acc[3];
    __syncthreads();
    if (threadIdx.x == 0 && i + kRing < nmine) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(i + kRing);
    }
    const float* rr = red + (size_t)(i & 1) * kWarps * kRows * kMaxT;
    for (int o = threadIdx.x; o < kRows * kMaxT; o += blockDim.x) {
      const int row = o / kMaxT, tok = o % kMaxT;
      if (tok >= p.T || r0 + row >= p.N) continue;
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; w++) v += rr[(size_t)w * kRows * kMaxT + o];
      if (p.ar_push) {      // row-parallel partial -> slot [rank] of every peer
        const size_t aoff = (size_t)tok * p.N + r0 + row;
        for (int q = 0; q < p.ar.world; q++) ar_slot(p.ar, q, epoch, p.ar.rank)[aoff] = v;
        continue;
      }
      const size_t off = (size_t)tok * p.out_stride + r0 + row;
      if (p.resid) v += __bfloat162float(p.resid[off]);
      if (p.out_f32) reinterpret_cast<float*>(p.out)[off] = v;
      else reinterpret_cast<__nv_bfloat16*>(p.out)[off] = __float2bfloat16(v);
    }
  }
  if (p.ar_push) ar_producer_arrive(p.ar, epoch);
}

}  // namespace moet

using namespace moet;

// Same contract as gemv_fp8 for unbatched weights, T <= 8, K % 64 == 0, K <= 8192.
void gemv_stream_fp8(c10::optional<torch::Tensor> a_opt, c10::optional<torch::Tensor> sa_opt, torch::Tensor w,
                     torch::Tensor sw, torch::Tensor out, c10::optional<torch::Tensor> resid, torch::Tensor status,
                     c10::optional<torch::Tensor> x_norm, c10::optional<torch::Tensor> gamma, double eps,
                     c10::optional<torch::Tensor> x_add, c10::optional<torch::Tensor> x_out,
                     c10::optional<torch::Tensor> ar_push, c10::optional<torch::Tensor> ar_consume) {
  const bool fuse = x_norm.has_value() && x_norm->defined();
  const torch::Tensor& a = fuse ? *x_norm : *a_opt;
  const int T = a.size(0), K = w.size(1), N = w.size(0);
  TORCH_CHECK(w.dim() == 2 && w.is_contiguous() && K % 128 == 0 && K <= gs::kMaxK && T <= gs::kMaxT,
              "gemv_stream_fp8: W [N, K] contiguous, K % 128 == 0, K <= 8192, T <= 8");
  TORCH_CHECK(a.size(1) == K && a.stride(1) == 1 && (a.stride(0) * a.element_size()) % 16 == 0, "gemv_stream_fp8: A");
  if (fuse) {
    TORCH_CHECK(a.scalar_type() == at::kBFloat16 && gamma.has_value() && gamma->numel() == K &&
                gamma->scalar_type() == at::kBFloat16 && gamma->is_contiguous(),
                "gemv_stream_fp8: fused norm needs bf16 x and a bf16 gamma of K");
  } else {
    TORCH_CHECK(sa_opt.has_value() && sa_opt->stride(1) == 1, "gemv_stream_fp8: activation scales");
  }
  TORCH_CHECK(reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0,
              "gemv_stream_fp8: 16-byte aligned operands");
  TORCH_CHECK(out.stride(1) == 1 && (out.scalar_type() == at::kFloat || out.scalar_type() == at::kBFloat16),
              "gemv_stream_fp8: out bf16 or f32");
  if (T == 0) return;
  GemvStreamArgs p;
  p.A = fuse ? nullptr : (const uint8_t*)a.data_ptr(); p.a_stride = fuse ? 0 : a.stride(0);
  p.sA = fuse ? nullptr : (const uint8_t*)sa_opt->data_ptr(); p.sa_stride = fuse ? 0 : sa_opt->stride(0);
  p.xin = fuse ? (const __nv_bfloat16*)a.data_ptr() : nullptr; p.xin_stride = fuse ? a.stride(0) : 0;
  p.gamma = fuse ? (const __nv_bfloat16*)gamma->data_ptr() : nullptr; p.eps = (float)eps;
  p.xadd = nullptr; p.xout = nullptr; p.xadd_stride = 0;
  if (fuse && x_add.has_value() && x_add->defined()) {
    TORCH_CHECK(x_add->scalar_type() == at::kBFloat16 && x_add->stride(1) == 1 && x_add->size(1) == K &&
                x_out.has_value() && x_out->is_contiguous() && x_out->size(1) == K, "gemv_stream_fp8: x_add / x_out");
    p.xadd = (const __nv_bfloat16*)x_add->data_ptr(); p.xadd_stride = x_add->stride(0);
    p.xout = (__nv_bfloat16*)x_out->data_ptr();
  }
  p.ar_push = ar_push.has_value() && ar_push->defined();
  p.ar_consume = ar_consume.has_value() && ar_consume->defined();
  p.ar = ArDesc{};
  if (p.ar_push) {
    p.ar = ar_desc_from(*ar_push);
    TORCH_CHECK((int64_t)T * N <= p.ar.cap, "gemv_stream_fp8: T*N exceeds the all-reduce slot");
  }
  if (p.ar_consume) {
    TORCH_CHECK(fuse && !p.xadd && x_out.has_value() && x_out->is_contiguous() && x_out->size(1) == K &&
                a.stride(0) == K && !p.ar_push, "gemv_stream_fp8: all-reduce consumer needs the fused norm, "
                "a contiguous residual and x_out");
    p.ar = ar_desc_from(*ar_consume);
    TORCH_CHECK((int64_t)T * K <= p.ar.cap, "gemv_stream_fp8: T*K exceeds the all-reduce slot");
    p.xout = (__nv_bfloat16*)x_out->data_ptr();
  }
  p.W = (const uint8_t*)w.data_ptr(); p.sW = (const uint8_t*)sw.data_ptr(); p.sw_cols = sw.size(1);
  p.out = out.data_ptr(); p.out_stride = out.stride(0); p.out_f32 = out.scalar_type() == at::kFloat;
  p.resid = resid.has_value() && resid->defined() ? (const __nv_bfloat16*)resid->data_ptr() : nullptr;
  if (p.resid) TORCH_CHECK(resid->stride(0) == out.stride(0), "gemv_stream_fp8: resid layout");
  p.T = T; p.N = N; p.K = K; p.status = status.data_ptr<int>();
  const int KP = K + 16;
  const size_t fixed = (size_t)gs::kMaxT * KP + (size_t)2 * gs::kWarps * gs::kRows * gs::kMaxT * 4 +
                       (size_t)gs::kMaxT * (gs::kMaxK / 64) * 4 + gs::kMaxRing * 8;
  const size_t budget = 220 * 1024;
  const int ring = (int)std::min<size_t>(gs::kMaxRing, (budget - fixed) / ((size_t)gs::kRows * KP));
  TORCH_CHECK(ring >= 2, "gemv_stream_fp8: K too large for a 2-stage ring");
  p.ring = ring;
  const size_t smem = (size_t)ring * gs::kRows * KP + fixed;
  static int n_sm = 0;
  if (!n_sm) cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, 0);
  const int nblocks = (N + gs::kRows - 1) / gs::kRows;
  moet_allow_max_smem(gemv_stream_kernel);
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_k(gemv_stream_kernel, std::min(nblocks, n_sm), gs::kWarps * 32, smem, stream, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
