// 2-bit sign-symmetric codebook expert GEMV/GEMM over a device pair list.
//
//   out[row_s, n] = sum_k A[row_s, k] * W_e[n, k]      for every pair (e, rows)
//
// W_e is a fragment-major plane of 2-bit codes {-4,-1,+1,+4} with UE8M0
// block-32 scales (the pack format), located through an expert -> slot
// table into a slot pool (fully resident weights use the identity table;
// the residency tiers remap slots).  A is FP8 e4m3 in the "w2 layout" with
// per-64 UE8M0 scales.  This is the B200 counterpart of the reference's
// moe_w2_mm SASS kernels (kernels/MANIFEST.md:104-148; ABI at P:6763-6775),
// written from the format specification:
//
// * Each warp owns one 16-row block of W; every lane streams 8 bytes
//   (32 codes) per 64-k chunk -- its MMA A-fragments for two k32 steps.
// * Decode: the codes of byte pairs sit at 4-bit strides, so
//   (w >> s) & 0x3333 is directly a prmt selector; one prmt over two
//   4-entry e4m3 lookup words (k32 half a in the low word, half b in the
//   high word, selected by bit 2 of each selector nibble) yields four e4m3
//   weights.  11 ALU ops decode 16 weights.
// * Scale folding: per row and 64-chunk the larger of the two block
//   exponents E is factored out; each k32 block's weights are encoded as
//   level * 2^(e - E) in e4m3 (exact down to 2^-9 relative; blocks more
//   than 2^9 smaller than their neighbour contribute < 2^-9 of it and are
//   flushed), so both MMAs accumulate into one fragment and the epilogue
//   applies 2^E * a_scale once per chunk.
// * Misses (slot < 0) write zero rows and bump a miss counter.
#include "common.cuh"
#include "torch_glue.h"

namespace moet {

// lut[m] = e4m3 bytes of {-4,-1,+1,+4} * 2^-m, code order, little-endian.
MOET_DEVICE uint8_t e4m3_pow2(int p, bool neg) {  // +-2^p as e4m3 (0 if underflow)
  uint8_t b;
  if (p >= -6) b = (uint8_t)((p + 7) << 3);
  else if (p >= -9) b = (uint8_t)(1 << (p + 9));
  else return 0;
  return neg ? (uint8_t)(b | 0x80) : b;
}
MOET_DEVICE uint32_t code_lut_word(int m) {
  return (uint32_t)e4m3_pow2(2 - m, true) | ((uint32_t)e4m3_pow2(-m, true) << 8) |
         ((uint32_t)e4m3_pow2(-m, false) << 16) | ((uint32_t)e4m3_pow2(2 - m, false) << 24);
}

struct W2Args {
  const uint8_t* A; const uint8_t* sA; long long a_stride;  // activations (w2 layout), row stride bytes
  const int* gather;            // sorted row -> activation row (nullptr: identity)
  const int4* pairs; const int* n_pairs;
  const uint8_t* pool; long long slot_bytes; long long codes_off, scale_off;
  const int* slot_table;        // expert -> slot (< 0: miss)
  float* out; long long out_stride;
  int N, K;
  int* miss_count;
};

template <int NT>
__global__ void __launch_bounds__(128) moe_w2_gemv_kernel(W2Args p) {
  __shared__ uint32_t lut[16];
  if (threadIdx.x < 16) lut[threadIdx.x] = code_lut_word(threadIdx.x);
  __syncthreads();
  const int pi = blockIdx.y;
  if (pi >= *p.n_pairs) return;
  const int4 pr = p.pairs[pi];
  const int e = pr.x, r0 = pr.y, nrows = pr.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int nb = blockIdx.x * (blockDim.x >> 5) + warp;  // 16-row block
  if (nb * 16 >= p.N) return;
  const int slot = p.slot_table[e];
  if (slot < 0) {
    if (blockIdx.x == 0 && threadIdx.x == 0 && p.miss_count) atomicAdd(p.miss_count, 1);
    for (int j = 0; j < nrows; j++)
      if (lane < 16) p.out[(size_t)(r0 + j) * p.out_stride + nb * 16 + lane] = 0.f;
    return;
  }
  const int KC = p.K >> 6, KS = p.K >> 5;
  const uint8_t* base = p.pool + (size_t)slot * p.slot_bytes;
  const uint8_t* codes = base + p.codes_off + (size_t)nb * KC * 256 + lane * 8;
  const uint8_t* sc = base + p.scale_off + (size_t)nb * KS * 16;

  // activation row of sorted row r0 + j (gathered through the token map for w13)
  auto act_row = [&](int j) -> int {
    const int r = r0 + min(j, nrows - 1);
    return p.gather ? __ldg(p.gather + r) : r;
  };
  int xr[NT], sr0[NT], sr1[NT];
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    xr[nt] = nt * 8 + g < nrows ? act_row(nt * 8 + g) : -1;
    sr0[nt] = nt * 8 + 2 * t < nrows ? act_row(nt * 8 + 2 * t) : -1;
    sr1[nt] = nt * 8 + 2 * t + 1 < nrows ? act_row(nt * 8 + 2 * t + 1) : -1;
  }
  const uint8_t* xbase = p.A + 8 * t;
  const int KC64 = p.K >> 6;
  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

#pragma unroll 4
  for (int c = 0; c < KC; c++) {
    const uint2 w = ldg_stream_u2(codes + (size_t)c * 256);
    const uint8_t* s = sc + (size_t)c * 32;
    const int ega = __ldg(s + g), eha = __ldg(s + g + 8), egb = __ldg(s + 16 + g), ehb = __ldg(s + 24 + g);
    const int Eg = max(ega, egb), Eh = max(eha, ehb);
    const uint32_t Lga = lut[min(Eg - ega, 15)], Lgb = lut[min(Eg - egb, 15)];
    const uint32_t Lha = lut[min(Eh - eha, 15)], Lhb = lut[min(Eh - ehb, 15)];
    const uint32_t lo = w.x, hi = w.y;
    uint32_t A0[4], A1[4];
    A0[0] = prmt(Lga, Lgb, lo & 0x3333u);
    A0[1] = prmt(Lha, Lhb, hi & 0x3333u);
    A0[2] = prmt(Lga, Lgb, (lo >> 2) & 0x3333u);
    A0[3] = prmt(Lha, Lhb, (hi >> 2) & 0x3333u);
    A1[0] = prmt(Lga, Lgb, ((lo >> 16) & 0x3333u) | 0x4444u);
    A1[1] = prmt(Lha, Lhb, ((hi >> 16) & 0x3333u) | 0x4444u);
    A1[2] = prmt(Lga, Lgb, ((lo >> 18) & 0x3333u) | 0x4444u);
    A1[3] = prmt(Lha, Lhb, ((hi >> 18) & 0x3333u) | 0x4444u);
    const float sg = ue8m0_to_float(Eg), sh = ue8m0_to_float(Eh);
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
      uint2 xa = make_uint2(0, 0), xb = make_uint2(0, 0);
      if (xr[nt] >= 0) {
        const uint8_t* xp = xbase + (size_t)xr[nt] * p.a_stride + (size_t)c * 64;
        xa = __ldg(reinterpret_cast<const uint2*>(xp));
        xb = __ldg(reinterpret_cast<const uint2*>(xp + 32));
      }
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      mma_e4m3_16832(d, A0, xa.x, xa.y, d);
      mma_e4m3_16832(d, A1, xb.x, xb.y, d);
      const float as0 = sr0[nt] >= 0 ? ue8m0_to_float(__ldg(p.sA + (size_t)sr0[nt] * KC64 + c)) : 0.f;
      const float as1 = sr1[nt] >= 0 ? ue8m0_to_float(__ldg(p.sA + (size_t)sr1[nt] * KC64 + c)) : 0.f;
      acc[nt][0] = fmaf(d[0], sg * as0, acc[nt][0]);
      acc[nt][1] = fmaf(d[1], sg * as1, acc[nt][1]);
      acc[nt][2] = fmaf(d[2], sh * as0, acc[nt][2]);
      acc[nt][3] = fmaf(d[3], sh * as1, acc[nt][3]);
    }
  }
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int j = nt * 8 + 2 * t + (i & 1);
      if (j >= nrows) continue;
      const int row = nb * 16 + g + ((i & 2) ? 8 : 0);
      p.out[(size_t)(r0 + j) * p.out_stride + row] = acc[nt][i];
    }
}

// out[t, :] = resid[t] (+ shared[t]) + sum_j w[t, j] * y[pos_of[t*k + j], :]  (fixed j order)
__global__ void moe_combine_kernel(const float* __restrict__ y, const int* __restrict__ pos_of,
                                   const float* __restrict__ wts, int k, int H,
                                   const __nv_bfloat16* __restrict__ resid,
                                   const __nv_bfloat16* __restrict__ shared_out,
                                   __nv_bfloat16* __restrict__ out, float* __restrict__ out_f32) {
  const int tok = blockIdx.x;
  __shared__ int pos[32];
  __shared__ float w[32];
  if (threadIdx.x < k) {
    pos[threadIdx.x] = pos_of[tok * k + threadIdx.x];
    w[threadIdx.x] = wts[tok * k + threadIdx.x];
  }
  __syncthreads();
  for (int h = threadIdx.x * 4; h < H; h += blockDim.x * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < k; j++) {
      const float4 v = *reinterpret_cast<const float4*>(y + (size_t)pos[j] * H + h);
      acc.x = fmaf(w[j], v.x, acc.x); acc.y = fmaf(w[j], v.y, acc.y);
      acc.z = fmaf(w[j], v.z, acc.z); acc.w = fmaf(w[j], v.w, acc.w);
    }
    float r[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      if (shared_out) r[i] += __bfloat162float(shared_out[(size_t)tok * H + h + i]);
      if (resid) r[i] += __bfloat162float(resid[(size_t)tok * H + h + i]);
      if (out) out[(size_t)tok * H + h + i] = __float2bfloat16(r[i]);
      if (out_f32) out_f32[(size_t)tok * H + h + i] = r[i];
    }
  }
}

}  // namespace moet

using namespace moet;

void moe_w2_gemv(torch::Tensor a, torch::Tensor sa, c10::optional<torch::Tensor> gather, torch::Tensor pairs,
                 torch::Tensor n_pairs, torch::Tensor pool, int64_t codes_off, int64_t scale_off,
                 torch::Tensor slot_table, torch::Tensor out, int64_t N, int64_t K, int64_t rows_per_pair,
                 c10::optional<torch::Tensor> miss_count) {
  TORCH_CHECK(K % 64 == 0 && N % 16 == 0, "moe_w2_gemv: N % 16, K % 64");
  TORCH_CHECK(a.stride(1) == 1 && a.size(1) == K, "moe_w2_gemv: A [rows, K] inner-contiguous");
  TORCH_CHECK(sa.is_contiguous() && sa.size(1) == K / 64, "moe_w2_gemv: sA [rows, K/64]");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.stride(1) == 1, "moe_w2_gemv: out f32");
  TORCH_CHECK(pool.dim() == 2, "moe_w2_gemv: pool [slots, slot_bytes]");
  TORCH_CHECK(codes_off % 16 == 0 && scale_off % 16 == 0 && pool.stride(0) % 16 == 0, "moe_w2_gemv: alignment");
  W2Args p;
  p.A = (const uint8_t*)a.data_ptr(); p.sA = (const uint8_t*)sa.data_ptr(); p.a_stride = a.stride(0);
  p.gather = gather.has_value() && gather->defined() ? gather->data_ptr<int>() : nullptr;
  p.pairs = (const int4*)pairs.data_ptr<int>(); p.n_pairs = n_pairs.data_ptr<int>();
  p.pool = (const uint8_t*)pool.data_ptr(); p.slot_bytes = pool.stride(0);
  p.codes_off = codes_off; p.scale_off = scale_off;
  p.slot_table = slot_table.data_ptr<int>();
  p.out = out.data_ptr<float>(); p.out_stride = out.stride(0);
  p.N = N; p.K = K;
  p.miss_count = miss_count.has_value() && miss_count->defined() ? miss_count->data_ptr<int>() : nullptr;
  const int max_pairs = pairs.size(0);
  const int wpc = 4;
  dim3 grid((N / 16 + wpc - 1) / wpc, max_pairs);
  auto stream = at::cuda::getCurrentCUDAStream();
  switch (rows_per_pair) {
    case 8: moe_w2_gemv_kernel<1><<<grid, wpc * 32, 0, stream>>>(p); break;
    case 16: moe_w2_gemv_kernel<2><<<grid, wpc * 32, 0, stream>>>(p); break;
    case 32: moe_w2_gemv_kernel<4><<<grid, wpc * 32, 0, stream>>>(p); break;
    default: TORCH_CHECK(false, "moe_w2_gemv: rows_per_pair must be 8/16/32");
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void moe_combine(torch::Tensor y, torch::Tensor pos_of, torch::Tensor wts, c10::optional<torch::Tensor> resid,
                 c10::optional<torch::Tensor> shared_out, c10::optional<torch::Tensor> out,
                 c10::optional<torch::Tensor> out_f32) {
  const int T = wts.size(0), k = wts.size(1), H = y.size(1);
  TORCH_CHECK(H % 4 == 0 && k <= 32, "moe_combine: H % 4, k <= 32");
  if (T == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  moe_combine_kernel<<<T, 256, 0, stream>>>(y.data_ptr<float>(), pos_of.data_ptr<int>(), wts.data_ptr<float>(), k, H,
                                            (const __nv_bfloat16*)opt_ptr(resid), (const __nv_bfloat16*)opt_ptr(shared_out),
                                            (__nv_bfloat16*)opt_ptr(out), (float*)opt_ptr(out_f32));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
