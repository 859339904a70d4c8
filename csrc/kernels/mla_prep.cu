// MLA per-token preparation kernels (decode and prefill):
//   q_prep : q_b output [T, Hh*(nope+rope)] -> FP8(q_nope) for the W_uk^T absorb
//            GEMV and RoPE(q_rope) written next to the absorbed query.
//   kv_prep: kv_a output [T, kv_lora+rope] -> RMSNorm(c_kv), RoPE(k_rope), cache
//            write at slot_mapping[t] in the bf16 row layout or the 352-byte
//            NVFP4 row (reference layout P:7-19; write semantics P:57-115,
//            but an out-of-range slot is reported through *status instead of
//            trapping; negative slots are padding and skipped).
// RoPE is the rotate-half form on the rope dims with a precomputed
// cos/sin table [max_pos, rope/2] (f32).
#include "common.cuh"
#include "torch_glue.h"

namespace moet {

// grid T, block 32*WH: warp per head (looping heads).
__global__ void q_prep_kernel(const __nv_bfloat16* __restrict__ qb, long long qb_stride, int Hh, int nope, int rope,
                              const int* __restrict__ pos_of_tok, const float* __restrict__ cos_sin,
                              uint8_t* __restrict__ qn_q, uint8_t* __restrict__ qn_s,
                              __nv_bfloat16* __restrict__ qcat, long long qcat_tok_stride, int qcat_head_stride,
                              int rope_off, __nv_bfloat16* __restrict__ q_out /* optional [T,Hh,nope+rope] */) {
  pdl_entry();
  const int tok = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int pos = pos_of_tok[tok];
  const int half = rope / 2;
  const float* cs = cos_sin + (size_t)pos * rope;  // [cos(half) | sin(half)]
  for (int h = blockIdx.y * nw + warp; h < Hh; h += nw * gridDim.y) {
    const __nv_bfloat16* src = qb + (size_t)tok * qb_stride + (size_t)h * (nope + rope);
    // nope -> fp8, groups of 64; each lane handles nope/32 consecutive values
    if (qn_q) {
      const int per = nope / 32;  // 4 for nope=128
      float v[8];
      for (int i = 0; i < per; i++) v[i] = __bfloat162float(src[lane * per + i]);
      float amax = 0.f;
      for (int i = 0; i < per; i++) amax = fmaxf(amax, fabsf(v[i]));
      const int lanes_per_group = 64 / per;
      for (int o = 1; o < lanes_per_group; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const uint32_t e = ue8m0_for_amax(amax);
      const float inv = (e >= 1 && e <= 253) ? __uint_as_float((254u - e) << 23) : 0.f;
      uint8_t* dq = qn_q + ((size_t)tok * Hh + h) * nope + lane * per;
      for (int i = 0; i < per; i++) dq[i] = f32_to_e4m3(v[i] * inv);
      if ((lane % lanes_per_group) == 0) qn_s[((size_t)tok * Hh + h) * (nope / 64) + (lane * per) / 64] = (uint8_t)e;
    }
    if (q_out) {
      for (int i = lane; i < nope; i += 32) q_out[((size_t)tok * Hh + h) * (nope + rope) + i] = src[i];
    }
    // rope: pairs (i, i+half)
    for (int i = lane; i < half; i += 32) {
      const float x1 = __bfloat162float(src[nope + i]), x2 = __bfloat162float(src[nope + i + half]);
      const float c = cs[i], s = cs[half + i];
      const float y1 = x1 * c - x2 * s, y2 = x2 * c + x1 * s;
      if (qcat) {
        __nv_bfloat16* d = qcat + (size_t)tok * qcat_tok_stride + (size_t)h * qcat_head_stride + rope_off;
        d[i] = __float2bfloat16(y1); d[i + half] = __float2bfloat16(y2);
      }
      if (q_out) {
        __nv_bfloat16* d = q_out + ((size_t)tok * Hh + h) * (nope + rope) + nope;
        d[i] = __float2bfloat16(y1); d[i + half] = __float2bfloat16(y2);
      }
    }
  }
}

// grid T, block 128.  kva: [T, lat+rope] (row stride kva_stride).
__global__ void kv_prep_kernel(const __nv_bfloat16* __restrict__ kva, long long kva_stride, int lat, int rope,
                               const __nv_bfloat16* __restrict__ norm_w, float eps,
                               const int* __restrict__ pos_of_tok, const float* __restrict__ cos_sin,
                               const long long* __restrict__ slot_mapping, long long num_slots,
                               int cache_mode /*0 none, 1 bf16, 2 nvfp4*/, uint8_t* __restrict__ cache,
                               __nv_bfloat16* __restrict__ lat_out, __nv_bfloat16* __restrict__ rope_out,
                               uint8_t* __restrict__ lat_q, uint8_t* __restrict__ lat_s, int* __restrict__ status) {
  pdl_entry();
  const int tok = blockIdx.x;
  const __nv_bfloat16* src = kva + (size_t)tok * kva_stride;
  __shared__ float vals[1024];
  __shared__ float red[4];
  float ss = 0.f;
  for (int i = threadIdx.x; i < lat; i += blockDim.x) {
    const float v = __bfloat162float(src[i]);
    vals[i] = v; ss += v * v;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  const float tot = red[0] + red[1] + red[2] + red[3];
  const float rinv = rsqrtf(tot / (float)lat + eps);
  for (int i = threadIdx.x; i < lat; i += blockDim.x)
    vals[i] = __bfloat162float(__float2bfloat16(vals[i] * rinv * __bfloat162float(norm_w[i])));
  const int pos = pos_of_tok[tok];
  const int half = rope / 2;
  const float* cs = cos_sin + (size_t)pos * rope;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float x1 = __bfloat162float(src[lat + i]), x2 = __bfloat162float(src[lat + i + half]);
    const float c = cs[i], s = cs[half + i];
    vals[lat + i] = __bfloat162float(__float2bfloat16(x1 * c - x2 * s));
    vals[lat + i + half] = __bfloat162float(__float2bfloat16(x2 * c + x1 * s));
  }
  __syncthreads();
  if (lat_out)
    for (int i = threadIdx.x; i < lat; i += blockDim.x) lat_out[(size_t)tok * lat + i] = __float2bfloat16(vals[i]);
  if (rope_out)
    for (int i = threadIdx.x; i < rope; i += blockDim.x) rope_out[(size_t)tok * rope + i] = __float2bfloat16(vals[lat + i]);
  if (lat_q) {  // fp8 natural layout, groups of 64 (2 lanes... 128 threads x 4 values)
    for (int base = 0; base < lat; base += blockDim.x * 4) {
      const int k0 = base + threadIdx.x * 4;
      float v[4] = {0, 0, 0, 0};
      const bool valid = k0 < lat;
      if (valid) for (int i = 0; i < 4; i++) v[i] = vals[k0 + i];
      float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
      for (int o = 1; o < 16; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const uint32_t e = ue8m0_for_amax(amax);
      const float inv = (e >= 1 && e <= 253) ? __uint_as_float((254u - e) << 23) : 0.f;
      if (valid) {
        for (int i = 0; i < 4; i++) lat_q[(size_t)tok * lat + k0 + i] = f32_to_e4m3(v[i] * inv);
        if ((threadIdx.x & 15) == 0) lat_s[(size_t)tok * (lat / 64) + k0 / 64] = (uint8_t)e;
      }
    }
  }
  if (cache_mode == 0) return;
  const long long slot = slot_mapping[tok];
  if (slot < 0) return;  // padding token
  if (slot >= num_slots) { if (threadIdx.x == 0) set_status(status, kBadIndex); return; }
  if (cache_mode == 1) {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(cache) + (size_t)slot * 584;
    for (int i = threadIdx.x; i < lat + rope; i += blockDim.x) dst[i] = __float2bfloat16(vals[i]);
  } else {
    // NVFP4 352-byte row (lat must be 512, rope 64)
    uint8_t* dst = cache + (size_t)slot * 352;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (w == 0) {
      float x[16];
      for (int i = 0; i < 16; i++) x[i] = vals[lane * 16 + i];
      float amax = 0.f;
      for (int i = 0; i < 16; i++) amax = fmaxf(amax, fabsf(x[i]));
      const float sf = __fdiv_rn(amax, 6.0f);
      const uint8_t sfq = f32_to_e4m3(fminf(sf * 64.0f, 448.0f));
      __nv_fp8_e4m3 sv; *reinterpret_cast<uint8_t*>(&sv) = sfq;
      const float scale = float(sv) * 0.015625f;
      const float inv = scale > 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
      float q[16];
      for (int i = 0; i < 16; i++) q[i] = x[i] * inv;
      uint2 packed;
      packed.x = f32x8_to_e2m1x8(q);
      packed.y = f32x8_to_e2m1x8(q + 8);
      *reinterpret_cast<uint2*>(dst + lane * 8) = packed;
      dst[256 + lane] = sfq;
    } else if (w == 1 && lane < 16) {
      uint32_t out = 0;
      for (int i = 0; i < 4; i++) {
        const float r = fminf(fmaxf(vals[lat + lane * 4 + i], -448.f), 448.f);
        out |= (uint32_t)f32_to_e4m3(r) << (8 * i);
      }
      *reinterpret_cast<uint32_t*>(dst + 288 + lane * 4) = out;
    }
  }
}

}  // namespace moet

using namespace moet;

void q_prep(torch::Tensor qb, int64_t Hh, int64_t nope, int64_t rope, torch::Tensor pos_of_tok,
            torch::Tensor cos_sin, c10::optional<torch::Tensor> qn_q, c10::optional<torch::Tensor> qn_s,
            c10::optional<torch::Tensor> qcat, int64_t rope_off, c10::optional<torch::Tensor> q_out) {
  const int T = qb.size(0);
  TORCH_CHECK(nope % 64 == 0 && nope <= 256 && rope % 2 == 0, "q_prep: nope % 64 == 0, <= 256");
  if (T == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  long long qcs = 0; int qhs = 0;
  if (qcat.has_value() && qcat->defined()) { qcs = qcat->stride(0); qhs = qcat->stride(1); }
  const int warps = std::min<int>(8, Hh);
  launch_k(q_prep_kernel, dim3(T, (Hh + warps - 1) / warps), 32 * warps, 0, stream, (const __nv_bfloat16*)qb.data_ptr(), qb.stride(0), Hh, nope, rope,
                                               pos_of_tok.data_ptr<int>(), cos_sin.data_ptr<float>(),
                                               (uint8_t*)opt_ptr(qn_q), (uint8_t*)opt_ptr(qn_s),
                                               (__nv_bfloat16*)opt_ptr(qcat), qcs, qhs, (int)rope_off,
                                               (__nv_bfloat16*)opt_ptr(q_out));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void kv_prep(torch::Tensor kva, int64_t lat, int64_t rope, torch::Tensor norm_w, double eps, torch::Tensor pos_of_tok,
             torch::Tensor cos_sin, c10::optional<torch::Tensor> slot_mapping, int64_t cache_mode,
             c10::optional<torch::Tensor> cache, c10::optional<torch::Tensor> lat_out,
             c10::optional<torch::Tensor> rope_out, c10::optional<torch::Tensor> lat_q,
             c10::optional<torch::Tensor> lat_s, torch::Tensor status) {
  const int T = kva.size(0);
  TORCH_CHECK(lat + rope <= 1024 && lat % 64 == 0, "kv_prep: lat+rope <= 1024");
  if (cache_mode == 2) TORCH_CHECK(lat == 512 && rope == 64, "kv_prep: NVFP4 rows need 512 + 64");
  if (T == 0) return;
  long long num_slots = 0;
  if (cache_mode == 1) num_slots = cache->numel() / 584;
  if (cache_mode == 2) num_slots = cache->numel() / 352;
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_k(kv_prep_kernel, T, 128, 0, stream, (const __nv_bfloat16*)kva.data_ptr(), kva.stride(0), lat, rope,
                                         (const __nv_bfloat16*)norm_w.data_ptr(), (float)eps,
                                         pos_of_tok.data_ptr<int>(), cos_sin.data_ptr<float>(),
                                         cache_mode ? (const long long*)slot_mapping->data_ptr<int64_t>() : nullptr, num_slots,
                                         (int)cache_mode, (uint8_t*)opt_ptr(cache), (__nv_bfloat16*)opt_ptr(lat_out),
                                         (__nv_bfloat16*)opt_ptr(rope_out), (uint8_t*)opt_ptr(lat_q),
                                         (uint8_t*)opt_ptr(lat_s), status.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
