// MLA prefill attention (non-absorbed): per head, q = [q_nope | q_rope] (DN + 64),
// k = [k_nope (from kv_b) | k_rope (shared by all heads)] (DN + 64), v (DV).
// DN = 128 / DV = 128 (DeepSeek-V4 shape) or DN = 192 / DV = 256 (GLM-5.x shape).
// A CTA accumulates 128 value columns; with DV = 256 two CTAs share a head (each
// recomputes Q.K^T), which keeps the O accumulator at 64 registers per thread.
// Causal within each sequence of a varlen batch (cu_seqlens).  With a separate key
// batch (cu_seqlens_k) sequence i's nq queries are its LAST nq positions: query j sits at
// position nk - nq + j and sees keys [0, nk - nq + j] -- a chunk of a long prompt whose
// earlier positions' K/V come from the cache.  Flash-attention
// structure: a CTA owns 128 query rows of one head (8 warps x 16 rows), Q
// fragments stay in registers, K/V tiles of 64 keys are double-buffered in
// shared memory with cp.async, softmax is online in registers, P is reused
// as the A operand of P.V without a shared-memory round trip.
// Epilogue writes the FP8 (e4m3, UE8M0 per-64) operand of o_proj directly,
// and optionally bf16.
#include "common.cuh"
#include "torch_glue.h"

namespace moet {

constexpr int kDV = 128;  // value columns per CTA
constexpr int kBQ = 128, kBK = 64;
constexpr int kVS = 136;  // V smem row (bf16)

MOET_DEVICE void cp_async16(void* dst, const void* src, bool pred) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  const int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(sz));
}
MOET_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N> MOET_DEVICE void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

struct PrefillArgs {
  const __nv_bfloat16* q; long long q_tok_stride; int q_head_stride;     // [T, Hh, DN + 64]
  const __nv_bfloat16* kvb; long long kvb_tok_stride; int kvb_head_stride; // [T, Hh, DN + DV] = k_nope | v
  const __nv_bfloat16* kr; long long kr_tok_stride;                      // [T, 64]
  const int* cu_seqlens; const int* cu_seqlens_k; int nseq;   // cu_seqlens_k null: keys = queries
  int Hh, DV;
  float scale_log2;
  uint8_t* out_q; uint8_t* out_s; __nv_bfloat16* out_bf16;   // [T, Hh*DV]
};

template <int kDN>
__global__ void __launch_bounds__(256, 1) mla_prefill_kernel(PrefillArgs p) {
  constexpr int kD = kDN + 64;
  constexpr int kKS = kD + 8;   // K / Q smem row (bf16): an odd number of 16-byte units
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __nv_bfloat16* Ks = reinterpret_cast<__nv_bfloat16*>(smem_raw);   // [2][64][kKS]
  __nv_bfloat16* Vs = Ks + 2 * kBK * kKS;                             // [2][64][136]
  __nv_bfloat16* Qs = Vs + 2 * kBK * kVS;                             // [128][kKS]
  const int nvc = p.DV / kDV;
  const int qtile = blockIdx.x, h = blockIdx.y / nvc, vc = blockIdx.y % nvc, sq = blockIdx.z;
  const int vcol0 = vc * kDV;                                         // this CTA's value columns
  const int s0 = p.cu_seqlens[sq], n = p.cu_seqlens[sq + 1] - s0;          // queries
  const int* cuk = p.cu_seqlens_k ? p.cu_seqlens_k : p.cu_seqlens;
  const int sk0 = cuk[sq], nk = cuk[sq + 1] - sk0;                         // keys
  const int off = nk - n;                                                  // position of query 0
  const int q0 = qtile * kBQ;
  if (q0 >= n || off < 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;

  // Q tile -> smem
  for (int i = threadIdx.x; i < kBQ * (kD / 8); i += blockDim.x) {
    const int r = i / (kD / 8), c = (i % (kD / 8)) * 8;
    const int tok = q0 + r;
    cp_async16(Qs + r * kKS + c, p.q + (size_t)(s0 + min(tok, n - 1)) * p.q_tok_stride + (size_t)h * p.q_head_stride + c,
               tok < n);
  }
  cp_async_commit();
  auto load_kv = [&](int kt, int buf) {
    const int k0 = kt * kBK;
    __nv_bfloat16* kd = Ks + buf * kBK * kKS;
    __nv_bfloat16* vd = Vs + buf * kBK * kVS;
    for (int i = threadIdx.x; i < kBK * (kD / 8); i += blockDim.x) {
      const int r = i / (kD / 8), c = (i % (kD / 8)) * 8;
      const int tok = k0 + r;
      const int tt = sk0 + min(tok, nk - 1);
      const __nv_bfloat16* src = c < kDN ? p.kvb + (size_t)tt * p.kvb_tok_stride + (size_t)h * p.kvb_head_stride + c
                                         : p.kr + (size_t)tt * p.kr_tok_stride + (c - kDN);
      cp_async16(kd + r * kKS + c, src, tok < nk);
    }
    for (int i = threadIdx.x; i < kBK * (kDV / 8); i += blockDim.x) {
      const int r = i / (kDV / 8), c = (i % (kDV / 8)) * 8;
      const int tok = k0 + r;
      const int tt = sk0 + min(tok, nk - 1);
      cp_async16(vd + r * kVS + c,
                 p.kvb + (size_t)tt * p.kvb_tok_stride + (size_t)h * p.kvb_head_stride + kDN + vcol0 + c, tok < nk);
    }
  };
  const int nkt = min((off + q0 + kBQ + kBK - 1) / kBK, (nk + kBK - 1) / kBK);
  load_kv(0, 0);
  cp_async_commit();
  cp_async_wait<1>();
  __syncthreads();
  // Q fragments -> registers
  uint32_t qf[kD / 16][4];
#pragma unroll
  for (int kk = 0; kk < kD / 16; kk++)
    ldmatrix_x4(qf[kk], Qs + (size_t)(warp * 16 + (lane & 15)) * kKS + kk * 16 + (lane >> 4) * 8);

  float o[kDV / 8][4];
#pragma unroll
  for (int i = 0; i < kDV / 8; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const int qrow0 = q0 + warp * 16 + g, qrow1 = qrow0 + 8;      // query rows (epilogue)
  const int kpos0 = off + qrow0, kpos1 = kpos0 + 8;               // their positions (causal mask)

  for (int kt = 0; kt < nkt; kt++) {
    const int buf = kt & 1;
    if (kt + 1 < nkt) load_kv(kt + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const __nv_bfloat16* kb = Ks + buf * kBK * kKS;
    const __nv_bfloat16* vb = Vs + buf * kBK * kVS;
    const int k0 = kt * kBK;
    // skip fully-masked tiles for this warp's rows
    const bool warp_active = k0 <= off + q0 + warp * 16 + 15;
    if (warp_active) {
      float s[kBK / 8][4];
#pragma unroll
      for (int i = 0; i < kBK / 8; i++) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < kD / 16; kk++) {
#pragma unroll
        for (int np = 0; np < kBK / 16; np++) {
          uint32_t b[4];
          // matrices: keys [np*16 + 0..7] dims kk*16+{0,8}; keys [np*16+8..15] dims kk*16+{0,8}
          const int krow = np * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int kcol = kk * 16 + ((lane >> 3) & 1) * 8;
          ldmatrix_x4(b, kb + (size_t)krow * kKS + kcol);
          mma_bf16_16816(s[2 * np], qf[kk], b[0], b[1]);
          mma_bf16_16816(s[2 * np + 1], qf[kk], b[2], b[3]);
        }
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int i = 0; i < kBK / 8; i++) {
        const int kc = k0 + i * 8 + 2 * t;
        s[i][0] = (kc <= kpos0 && kc < nk) ? s[i][0] * p.scale_log2 : -INFINITY;
        s[i][1] = (kc + 1 <= kpos0 && kc + 1 < nk) ? s[i][1] * p.scale_log2 : -INFINITY;
        s[i][2] = (kc <= kpos1 && kc < nk) ? s[i][2] * p.scale_log2 : -INFINITY;
        s[i][3] = (kc + 1 <= kpos1 && kc + 1 < nk) ? s[i][3] * p.scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, fmaxf(s[i][0], s[i][1]));
        mx1 = fmaxf(mx1, fmaxf(s[i][2], s[i][3]));
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1)); mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1)); mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);
      const float al0 = mn0 == -INFINITY ? 1.f : exp2f(m_run[0] - mn0);
      const float al1 = mn1 == -INFINITY ? 1.f : exp2f(m_run[1] - mn1);
      m_run[0] = mn0; m_run[1] = mn1;
      float rs0 = 0.f, rs1 = 0.f;
      uint32_t pf[kBK / 16][4];
#pragma unroll
      for (int i = 0; i < kBK / 8; i++) {
        const float e0 = mn0 == -INFINITY ? 0.f : exp2f(s[i][0] - mn0);
        const float e1 = mn0 == -INFINITY ? 0.f : exp2f(s[i][1] - mn0);
        const float e2 = mn1 == -INFINITY ? 0.f : exp2f(s[i][2] - mn1);
        const float e3 = mn1 == -INFINITY ? 0.f : exp2f(s[i][3] - mn1);
        __nv_bfloat162 a = __floats2bfloat162_rn(e0, e1), b2 = __floats2bfloat162_rn(e2, e3);
        rs0 += __low2float(a) + __high2float(a);
        rs1 += __low2float(b2) + __high2float(b2);
        pf[i >> 1][(i & 1) * 2 + 0] = *reinterpret_cast<uint32_t*>(&a);
        pf[i >> 1][(i & 1) * 2 + 1] = *reinterpret_cast<uint32_t*>(&b2);
      }
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1); rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1); rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
      l_run[0] = l_run[0] * al0 + rs0;
      l_run[1] = l_run[1] * al1 + rs1;
#pragma unroll
      for (int i = 0; i < kDV / 8; i++) { o[i][0] *= al0; o[i][1] *= al0; o[i][2] *= al1; o[i][3] *= al1; }
      // pf[j] = {a0: row g k 2t (tile 2j), a1: row g+8 (tile 2j), a2: row g k 8+2t (tile 2j+1), a3}
#pragma unroll
      for (int j = 0; j < kBK / 16; j++) {
        const uint32_t a[4] = {pf[j][0], pf[j][1], pf[j][2], pf[j][3]};
#pragma unroll
        for (int np = 0; np < kDV / 16; np++) {
          uint32_t b[4];
          const int vrow = j * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int vcol = np * 16 + (lane >> 4) * 8;
          ldmatrix_x4_trans(b, vb + (size_t)vrow * kVS + vcol);
          mma_bf16_16816(o[2 * np], a, b[0], b[1]);
          mma_bf16_16816(o[2 * np + 1], a, b[2], b[3]);
        }
      }
    }
    __syncthreads();
  }
  // epilogue
  const float inv0 = l_run[0] > 0.f ? 1.f / l_run[0] : 0.f, inv1 = l_run[1] > 0.f ? 1.f / l_run[1] : 0.f;
  const int HD = p.Hh * p.DV;
  const int ocol0 = h * p.DV + vcol0;
#pragma unroll
  for (int hr = 0; hr < 2; hr++) {
    const int qr = hr ? qrow1 : qrow0;
    const float inv = hr ? inv1 : inv0;
    float v[kDV / 8][2];
#pragma unroll
    for (int i = 0; i < kDV / 8; i++) {
      v[i][0] = __bfloat162float(__float2bfloat16(o[i][2 * hr] * inv));
      v[i][1] = __bfloat162float(__float2bfloat16(o[i][2 * hr + 1] * inv));
    }
    const bool valid = qr < n;
    const size_t row = (size_t)(s0 + (valid ? qr : 0));
    if (p.out_bf16 && valid) {
#pragma unroll
      for (int i = 0; i < kDV / 8; i++)
        *reinterpret_cast<__nv_bfloat162*>(p.out_bf16 + row * HD + ocol0 + i * 8 + 2 * t) =
            __floats2bfloat162_rn(v[i][0], v[i][1]);
    }
    if (p.out_q) {
#pragma unroll
      for (int gi = 0; gi < kDV / 64; gi++) {
        float amax = 0.f;
#pragma unroll
        for (int i = gi * 8; i < gi * 8 + 8; i++) amax = fmaxf(amax, fmaxf(fabsf(v[i][0]), fabsf(v[i][1])));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        const uint32_t e = ue8m0_for_amax(amax);
        const float invs = (e >= 1 && e <= 253) ? __uint_as_float((254u - e) << 23) : 0.f;
        if (valid) {
#pragma unroll
          for (int i = gi * 8; i < gi * 8 + 8; i++) {
            const uint16_t b = (uint16_t)f32_to_e4m3(v[i][0] * invs) | ((uint16_t)f32_to_e4m3(v[i][1] * invs) << 8);
            *reinterpret_cast<uint16_t*>(p.out_q + row * HD + ocol0 + i * 8 + 2 * t) = b;
          }
          if (t == 0) p.out_s[row * (HD / 64) + ocol0 / 64 + gi] = (uint8_t)e;
        }
      }
    }
  }
}

}  // namespace moet

using namespace moet;

void mla_prefill(torch::Tensor q, torch::Tensor kvb, torch::Tensor kr, torch::Tensor cu_seqlens, int64_t max_len,
                 double scale, c10::optional<torch::Tensor> out_q, c10::optional<torch::Tensor> out_s,
                 c10::optional<torch::Tensor> out_bf16, c10::optional<torch::Tensor> cu_seqlens_k) {
  const int Hh = q.size(1);
  const int DN = q.size(2) - 64, DV = kvb.size(2) - DN;
  TORCH_CHECK((DN == 128 || DN == 192) && q.stride(2) == 1, "mla_prefill: q [T, Hh, 192 | 256] (nope 128 | 192 + rope 64)");
  TORCH_CHECK(DV % kDV == 0 && DV > 0 && DV <= 512 && kvb.stride(2) == 1, "mla_prefill: kvb [T, Hh, nope + v], v % 128");
  TORCH_CHECK(kr.size(1) == 64 && kr.stride(1) == 1, "mla_prefill: kr [T, 64]");
  const int nseq = cu_seqlens.size(0) - 1;
  if (nseq == 0 || max_len == 0) return;
  PrefillArgs p;
  p.q = (const __nv_bfloat16*)q.data_ptr(); p.q_tok_stride = q.stride(0); p.q_head_stride = q.stride(1);
  p.kvb = (const __nv_bfloat16*)kvb.data_ptr(); p.kvb_tok_stride = kvb.stride(0); p.kvb_head_stride = kvb.stride(1);
  p.kr = (const __nv_bfloat16*)kr.data_ptr(); p.kr_tok_stride = kr.stride(0);
  p.cu_seqlens = cu_seqlens.data_ptr<int>(); p.nseq = nseq; p.Hh = Hh; p.DV = DV;
  p.cu_seqlens_k = nullptr;
  if (cu_seqlens_k.has_value() && cu_seqlens_k->defined()) {
    TORCH_CHECK(cu_seqlens_k->numel() == nseq + 1 && cu_seqlens_k->scalar_type() == at::kInt && cu_seqlens_k->is_cuda(),
                "mla_prefill: cu_seqlens_k [nseq + 1] int32 on the device");
    p.cu_seqlens_k = cu_seqlens_k->data_ptr<int>();
  }
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  p.out_q = (uint8_t*)opt_ptr(out_q); p.out_s = (uint8_t*)opt_ptr(out_s); p.out_bf16 = (__nv_bfloat16*)opt_ptr(out_bf16);
  auto stream = at::cuda::getCurrentCUDAStream();
  dim3 grid((max_len + kBQ - 1) / kBQ, Hh * (DV / kDV), nseq);
  auto launch = [&](auto dn) {
    constexpr int kDN = decltype(dn)::value, kKS = kDN + 64 + 8;
    const size_t smem = (size_t)(2 * kBK * kKS + 2 * kBK * kVS + kBQ * kKS) * 2;
    moet_allow_max_smem(mla_prefill_kernel<kDN>);
    mla_prefill_kernel<kDN><<<grid, 256, smem, stream>>>(p);
  };
  if (DN == 128) launch(std::integral_constant<int, 128>{});
  else launch(std::integral_constant<int, 192>{});
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
