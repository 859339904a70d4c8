// Hyper-connections (DeepSeek-V4 mHC) on the GPU: the residual is NH streams per token,
// xs [T, NH, H] f32.  Around every block a site computes, from the RMS-scaled flattened
// streams, m = (flat . fn^T) / rms(flat) over R = (NH + 2) NH rows of fn, and from m
//   pre  = sigmoid(m[0:NH] s0 + b) + eps          block input  h = sum_i pre_i x_i
//   post = 2 sigmoid(m[NH:2NH] s1 + b)            weight of the block output per stream
//   comb = row softmax(m[2NH:] s2 + b) + eps, then Sinkhorn (column, then row/column
//          normalisations) -> doubly stochastic NH x NH mix
// and after the block  x'_j = sum_i comb_ij x_i + post_j out.  A head site (R = NH rows)
// gives gate = sigmoid(m s0 + b) + eps and h = sum_i gate_i x_i.
// (Reference model: the upstream DeepSeek-V4 decoder layer's hc_pre / hc_post and the
// head's stream reduction, which vLLM-Moet serves through upstream tilelang kernels,
// patch/vllm-moet-v0.24.0.patch:14507-14510, 14670-14680.)
//
// Two kernels per site:
//   hc_mix    grid (H / 128 column slices, token groups).  A thread owns one column of all
//             NH streams: it first applies the previous block's update (x' = comb^T x +
//             post * out, written back in place) when one is pending, then accumulates its
//             column's share of the R dot products and of sum(x^2); partial sums per
//             column slice go to part[slice][t][R + 1] (fixed order, deterministic).  fn's
//             column stays in registers across the CTA's tokens.  R = 0: update only.
//   hc_apply  grid T.  Sums the slices in order, computes the mixes (one thread; NH <= 4),
//             writes post / comb for the next hc_mix, and h = sum_i pre_i x_i (bf16) --
//             the input of the block's RMSNorm.
#include "common.cuh"
#include "torch_glue.h"

namespace moet {

constexpr int kHcCols = 128;   // columns per hc_mix CTA (one per thread)

MOET_DEVICE float hc_sigmoid(float z) { return 1.f / (1.f + expf(-z)); }

template <int NH, int R>
__global__ void __launch_bounds__(kHcCols) hc_mix_kernel(float* __restrict__ xs, int T, int H,
                                                          const __nv_bfloat16* __restrict__ upd,
                                                          const float* __restrict__ post,
                                                          const float* __restrict__ comb,
                                                          const float* __restrict__ fn, float* __restrict__ part,
                                                          int tok_per_cta) {
  constexpr int RW = R > 0 ? R : 1;
  const int col = blockIdx.x * kHcCols + threadIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float w[RW][NH];
  if constexpr (R > 0) {          // weights: immutable, read before the dependency wait
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int i = 0; i < NH; i++) w[r][i] = fn[(size_t)r * NH * H + (size_t)i * H + col];
  }
  pdl_entry();
  __shared__ float red[kHcCols / 32][RW + 1];
  const int t0 = blockIdx.y * tok_per_cta, t1 = min(T, t0 + tok_per_cta);
  for (int t = t0; t < t1; t++) {
    float x[NH];
#pragma unroll
    for (int i = 0; i < NH; i++) x[i] = xs[((size_t)t * NH + i) * H + col];
    if (upd != nullptr) {
      const float a = __bfloat162float(upd[(size_t)t * H + col]);
      float y[NH];
#pragma unroll
      for (int j = 0; j < NH; j++) {
        float v = post[t * NH + j] * a;
#pragma unroll
        for (int i = 0; i < NH; i++) v += comb[((size_t)t * NH + i) * NH + j] * x[i];
        y[j] = v;
      }
#pragma unroll
      for (int j = 0; j < NH; j++) {
        x[j] = y[j];
        xs[((size_t)t * NH + j) * H + col] = y[j];
      }
    }
    if constexpr (R > 0) {
      float acc[R + 1];
      acc[R] = 0.f;
#pragma unroll
      for (int i = 0; i < NH; i++) acc[R] += x[i] * x[i];
#pragma unroll
      for (int r = 0; r < R; r++) {
        float v = 0.f;
#pragma unroll
        for (int i = 0; i < NH; i++) v += w[r][i] * x[i];
        acc[r] = v;
      }
#pragma unroll
      for (int r = 0; r <= R; r++) {
        float v = acc[r];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[warp][r] = v;
      }
      __syncthreads();
      if (threadIdx.x <= R) {
        float s = 0.f;
#pragma unroll
        for (int q = 0; q < kHcCols / 32; q++) s += red[q][threadIdx.x];
        part[((size_t)blockIdx.x * T + t) * (R + 1) + threadIdx.x] = s;
      }
      __syncthreads();
    }
  }
}

template <int NH>
__global__ void __launch_bounds__(256) hc_apply_kernel(const float* __restrict__ xs, int T, int H,
                                                        const float* __restrict__ part, int KS, int R,
                                                        const float* __restrict__ base,
                                                        const float* __restrict__ scale, float eps, int iters,
                                                        float rms_eps, __nv_bfloat16* __restrict__ h,
                                                        float* __restrict__ post, float* __restrict__ comb) {
  pdl_entry();
  const int t = blockIdx.x;
  __shared__ float m[(NH + 2) * NH + 1];
  __shared__ float pre[NH];
  for (int r = threadIdx.x; r <= R; r += blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < KS; k++) s += part[((size_t)k * T + t) * (R + 1) + r];
    m[r] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const float inv = rsqrtf(m[R] / (float)(NH * H) + rms_eps);
#pragma unroll
    for (int i = 0; i < NH; i++) pre[i] = hc_sigmoid(m[i] * inv * scale[0] + base[i]) + eps;
    if (post != nullptr) {
#pragma unroll
      for (int j = 0; j < NH; j++) post[t * NH + j] = 2.f * hc_sigmoid(m[NH + j] * inv * scale[1] + base[NH + j]);
      float c[NH][NH];
#pragma unroll
      for (int i = 0; i < NH; i++) {
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < NH; j++) {
          c[i][j] = m[2 * NH + i * NH + j] * inv * scale[2] + base[2 * NH + i * NH + j];
          mx = fmaxf(mx, c[i][j]);
        }
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < NH; j++) { c[i][j] = expf(c[i][j] - mx); s += c[i][j]; }
#pragma unroll
        for (int j = 0; j < NH; j++) c[i][j] = c[i][j] / s + eps;
      }
      auto col_norm = [&]() {
#pragma unroll
        for (int j = 0; j < NH; j++) {
          float s = 0.f;
#pragma unroll
          for (int i = 0; i < NH; i++) s += c[i][j];
#pragma unroll
          for (int i = 0; i < NH; i++) c[i][j] /= s + eps;
        }
      };
      col_norm();
      for (int it = 1; it < iters; it++) {
#pragma unroll
        for (int i = 0; i < NH; i++) {
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < NH; j++) s += c[i][j];
#pragma unroll
          for (int j = 0; j < NH; j++) c[i][j] /= s + eps;
        }
        col_norm();
      }
#pragma unroll
      for (int i = 0; i < NH; i++)
#pragma unroll
        for (int j = 0; j < NH; j++) comb[((size_t)t * NH + i) * NH + j] = c[i][j];
    }
  }
  __syncthreads();
  for (int col = threadIdx.x; col < H; col += blockDim.x) {
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < NH; i++) v += pre[i] * xs[((size_t)t * NH + i) * H + col];
    h[(size_t)t * H + col] = __float2bfloat16(v);
  }
}

}  // namespace moet

using namespace moet;

namespace {
void check_streams(const torch::Tensor& xs, int& T, int& NH, int& H) {
  TORCH_CHECK(xs.is_cuda() && xs.scalar_type() == at::kFloat && xs.dim() == 3 && xs.is_contiguous(),
              "hyper-connections: xs [T, n, H] f32 contiguous");
  T = xs.size(0); NH = xs.size(1); H = xs.size(2);
  TORCH_CHECK(NH == 2 || NH == 4, "hyper-connections: n = 2 or 4 streams");
  TORCH_CHECK(H % kHcCols == 0, "hyper-connections: hidden % 128");
}
}  // namespace

// xs updated in place when `upd` is given (x' = comb^T x + post * upd); partial mixes of fn's
// rows into part [H / 128, T, R + 1] when fn is given.
void hc_mix(torch::Tensor xs, c10::optional<torch::Tensor> upd, c10::optional<torch::Tensor> post,
            c10::optional<torch::Tensor> comb, c10::optional<torch::Tensor> fn, c10::optional<torch::Tensor> part) {
  int T, NH, H;
  check_streams(xs, T, NH, H);
  const bool has_upd = upd.has_value() && upd->defined(), has_fn = fn.has_value() && fn->defined();
  if (has_upd) {
    TORCH_CHECK(upd->scalar_type() == at::kBFloat16 && upd->is_contiguous() && upd->numel() == (int64_t)T * H,
                "hc_mix: upd [T, H] bf16");
    TORCH_CHECK(post.has_value() && post->scalar_type() == at::kFloat && post->is_contiguous() &&
                post->numel() >= (int64_t)T * NH, "hc_mix: post [T, n] f32");
    TORCH_CHECK(comb.has_value() && comb->scalar_type() == at::kFloat && comb->is_contiguous() &&
                comb->numel() >= (int64_t)T * NH * NH, "hc_mix: comb [T, n, n] f32");
  }
  int R = 0;
  const int KS = H / kHcCols;
  if (has_fn) {
    TORCH_CHECK(fn->scalar_type() == at::kFloat && fn->is_contiguous() && fn->dim() == 2 && fn->size(1) == NH * H,
                "hc_mix: fn [R, n H] f32");
    R = fn->size(0);
    TORCH_CHECK(R == NH || R == (NH + 2) * NH, "hc_mix: fn rows n (head) or (n + 2) n (block)");
    TORCH_CHECK(part.has_value() && part->scalar_type() == at::kFloat && part->is_contiguous() &&
                part->numel() >= (int64_t)KS * T * (R + 1), "hc_mix: part [H / 128, T, R + 1] f32");
  }
  if (T == 0 || (!has_upd && !has_fn)) return;
  const int tok = T >= 1024 ? 8 : 1;
  dim3 grid(KS, (T + tok - 1) / tok);
  auto stream = at::cuda::getCurrentCUDAStream();
  float* xp = xs.data_ptr<float>();
  auto* up = has_upd ? (const __nv_bfloat16*)upd->data_ptr() : nullptr;
  const float* pp = has_upd ? post->data_ptr<float>() : nullptr;
  const float* cp = has_upd ? comb->data_ptr<float>() : nullptr;
  const float* fp = has_fn ? fn->data_ptr<float>() : nullptr;
  float* qp = has_fn ? part->data_ptr<float>() : nullptr;
#define HC_MIX(NH_, R_) launch_k(hc_mix_kernel<NH_, R_>, grid, kHcCols, 0, stream, xp, T, H, up, pp, cp, fp, qp, tok)
  if (NH == 2) {
    if (R == 0) HC_MIX(2, 0); else if (R == 2) HC_MIX(2, 2); else HC_MIX(2, 8);
  } else {
    if (R == 0) HC_MIX(4, 0); else if (R == 4) HC_MIX(4, 4); else HC_MIX(4, 24);
  }
#undef HC_MIX
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// From hc_mix's partials: the site's mixes and h = sum_i pre_i x_i (bf16 [T, H]).  post /
// comb given: a block site (writes them); absent: a head site (gate = pre).
void hc_apply(torch::Tensor xs, torch::Tensor part, torch::Tensor base, torch::Tensor scale, double eps,
              int64_t iters, double rms_eps, torch::Tensor h, c10::optional<torch::Tensor> post,
              c10::optional<torch::Tensor> comb) {
  int T, NH, H;
  check_streams(xs, T, NH, H);
  const bool block = post.has_value() && post->defined();
  const int R = block ? (NH + 2) * NH : NH;
  const int KS = H / kHcCols;
  TORCH_CHECK(part.scalar_type() == at::kFloat && part.is_contiguous() && part.numel() >= (int64_t)KS * T * (R + 1),
              "hc_apply: part [H / 128, T, R + 1] f32");
  TORCH_CHECK(base.scalar_type() == at::kFloat && base.is_cuda() && base.numel() == R, "hc_apply: base [R] f32");
  TORCH_CHECK(scale.scalar_type() == at::kFloat && scale.is_cuda() && scale.numel() == (block ? 3 : 1),
              "hc_apply: scale [3 | 1] f32");
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && h.is_contiguous() && h.numel() == (int64_t)T * H, "hc_apply: h [T, H] bf16");
  if (block)
    TORCH_CHECK(post->scalar_type() == at::kFloat && post->is_contiguous() && post->numel() >= (int64_t)T * NH &&
                comb.has_value() && comb->scalar_type() == at::kFloat && comb->is_contiguous() &&
                comb->numel() >= (int64_t)T * NH * NH, "hc_apply: post [T, n], comb [T, n, n] f32");
  TORCH_CHECK(iters >= 1, "hc_apply: iters >= 1");
  if (T == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  float* pp = block ? post->data_ptr<float>() : nullptr;
  float* cp = block ? comb->data_ptr<float>() : nullptr;
  auto* hp = (__nv_bfloat16*)h.data_ptr();
  if (NH == 2)
    launch_k(hc_apply_kernel<2>, T, 256, 0, stream, (const float*)xs.data_ptr<float>(), T, H,
             (const float*)part.data_ptr<float>(), KS, R, (const float*)base.data_ptr<float>(),
             (const float*)scale.data_ptr<float>(), (float)eps, (int)iters, (float)rms_eps, hp, pp, cp);
  else
    launch_k(hc_apply_kernel<4>, T, 256, 0, stream, (const float*)xs.data_ptr<float>(), T, H,
             (const float*)part.data_ptr<float>(), KS, R, (const float*)base.data_ptr<float>(),
             (const float*)scale.data_ptr<float>(), (float)eps, (int)iters, (float)rms_eps, hp, pp, cp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
