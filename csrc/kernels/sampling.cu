// Sampling-side kernels of the decode step.
//   argmax_lse : per row argmax (ties -> lowest id) and log-sum-exp of the logits;
//                max_prob = exp(max - lse) is the confidence-gate signal
//                (reference gate P:11554-11628).
//   mtp_accept : greedy verification of k MTP drafts: accepted = longest prefix with
//                draft[j] == target[j]; emits target[0..accepted]; reports per-row
//                acceptance.  All state stays on the device (graph-replayable).
//   mtp_finalize: advances the per-sequence position and builds the next step's
//                 input tokens [target[a], draft_1 .. draft_k].
#include "common.cuh"
#include "symm.cuh"
#include "torch_glue.h"

namespace moet {

template <typename T>
__global__ void argmax_lse_kernel(const T* __restrict__ logits, long long stride, int V,
                                  int* __restrict__ ids, float* __restrict__ lse, float* __restrict__ maxv,
                                  int* __restrict__ status) {
  pdl_entry();
  const int row = blockIdx.x;
  const T* x = logits + (size_t)row * stride;
  float bv = -INFINITY; int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = (float)x[i];
    if (v > bv) { bv = v; bi = i; }
  }
  __shared__ float sv[32]; __shared__ int si[32]; __shared__ float ssum[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o); const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (l == 0) { sv[w] = bv; si[w] = bi; }
  __syncthreads();
  if (w == 0) {
    bv = l < nw ? sv[l] : -INFINITY; bi = l < nw ? si[l] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o); const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (l == 0) { sv[0] = bv; si[0] = bi; }
  }
  __syncthreads();
  const float m = sv[0];
  if (lse) {
    float s = 0.f;
    for (int i = threadIdx.x; i < V; i += blockDim.x) s += __expf((float)x[i] - m);
    s = warp_sum(s);
    if (l == 0) ssum[w] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
      float tot = 0.f;
      for (int i = 0; i < nw; i++) tot += ssum[i];
      lse[row] = m + __logf(tot);
    }
  }
  if (threadIdx.x == 0) {
    int id = si[0];
    if (id < 0 || id >= V) { id = 0; set_status(status, kBadValue); }  // no finite logit
    ids[row] = id;
    if (maxv) maxv[row] = m;
  }
}

// targets [B, 1+k] (argmax of the verify rows), tokens [B, 1+k] (this step's inputs;
// cols 1..k are the drafts).  out_tokens [B, 1+k], n_acc [B].
__global__ void mtp_accept_kernel(const int* __restrict__ targets, const int* __restrict__ tokens, int B, int kp1,
                                  int* __restrict__ out_tokens, int* __restrict__ n_acc,
                                  const int* __restrict__ active) {
  pdl_entry();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  int a = 0;
  if (!active || active[b]) {
    while (a + 1 < kp1 && tokens[b * kp1 + a + 1] == targets[b * kp1 + a]) a++;
  }
  for (int j = 0; j < kp1; j++) out_tokens[b * kp1 + j] = j <= a ? targets[b * kp1 + j] : -1;
  n_acc[b] = a;
}

// next inputs: tokens[b] = [targets[b, a], drafts[b, 0..k-1]]; seq_pos[b] += a + 1.
__global__ void mtp_finalize_kernel(const int* __restrict__ targets, const int* __restrict__ n_acc,
                                    const int* __restrict__ drafts, int B, int kp1, int* __restrict__ tokens,
                                    int* __restrict__ seq_pos, const int* __restrict__ active) {
  pdl_entry();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  if (active && !active[b]) return;
  const int a = n_acc[b];
  tokens[b * kp1] = targets[b * kp1 + a];
  for (int j = 1; j < kp1; j++) tokens[b * kp1 + j] = drafts[b * (kp1 - 1) + (j - 1)];
  seq_pos[b] += a + 1;
}

// Split argmax (+ optional log-sum-exp): grid (rows, S).  Each block reduces
// its slice to (max, argmax, sum exp(x - max)) in `part`; the last block of a
// row (per-row arrival counter) merges the S partials and resets the counter,
// so the kernel is replayable inside a CUDA graph.
template <typename T>
__global__ void argmax_split_kernel(const T* __restrict__ logits, long long stride, int V, int want_lse,
                                    float* __restrict__ part, int* __restrict__ counter, int* __restrict__ ids,
                                    float* __restrict__ lse, int* __restrict__ status,
                                    float2* __restrict__ mv = nullptr, int id_offset = 0) {
  pdl_entry();
  const int row = blockIdx.x, S = gridDim.y, sp = blockIdx.y;
  const int per = (V + S - 1) / S, lo = sp * per, hi = min(V, lo + per);
  const T* x = logits + (size_t)row * stride;
  float bv = -INFINITY; int bi = 0x7fffffff;
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const float v = (float)x[i];
    if (v > bv) { bv = v; bi = i; }
  }
  __shared__ float sv[32]; __shared__ int si[32]; __shared__ float ssum[32]; __shared__ int last;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o); const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  if (l == 0) { sv[w] = bv; si[w] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < nw; i++)
      if (sv[i] > sv[0] || (sv[i] == sv[0] && si[i] < si[0])) { sv[0] = sv[i]; si[0] = si[i]; }
  }
  __syncthreads();
  const float m = sv[0];
  float sum = 0.f;
  if (want_lse && m != -INFINITY) {
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) sum += __expf((float)x[i] - m);
    sum = warp_sum(sum);
    if (l == 0) ssum[w] = sum;
    __syncthreads();
    if (threadIdx.x == 0) { float t = 0.f; for (int i = 0; i < nw; i++) t += ssum[i]; sum = t; }
  }
  if (threadIdx.x == 0) {
    float* pp = part + ((size_t)row * S + sp) * 3;
    pp[0] = m; pp[1] = __int_as_float(si[0]); pp[2] = sum;
    __threadfence();
    last = atomicAdd(&counter[row], 1) == S - 1;
  }
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  __threadfence();
  float M = -INFINITY; int I = 0x7fffffff;
  for (int j = 0; j < S; j++) {
    const volatile float* pp = part + ((size_t)row * S + j) * 3;
    const float v = pp[0]; const int id = __float_as_int(pp[1]);
    if (v > M || (v == M && id < I)) { M = v; I = id; }
  }
  if (want_lse) {
    float tot = 0.f;
    for (int j = 0; j < S; j++) {
      const volatile float* pp = part + ((size_t)row * S + j) * 3;
      if (pp[0] != -INFINITY) tot += __expf(pp[0] - M) * pp[2];
    }
    lse[row] = M + __logf(tot);
  }
  if (I < 0 || I >= V) { I = 0; set_status(status, kBadValue); }
  if (ids) ids[row] = I + id_offset;
  if (mv) mv[row] = make_float2(M, __int_as_float(I + id_offset));
  counter[row] = 0;
}

// Vocab-parallel argmax merge: parts [W, R] of (max, id bits) from W ranks (ids
// already global) -> ids[R]; ties go to the smaller id, as in the 1-rank argmax.
__global__ void argmax_merge_kernel(const float2* __restrict__ parts, int W, int R, int* __restrict__ ids) {
  pdl_entry();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= R) return;
  float M = -INFINITY; int I = 0x7fffffff;
  for (int w = 0; w < W; w++) {
    const float2 p = parts[(size_t)w * R + r];
    const int id = __float_as_int(p.y);
    if (p.x > M || (p.x == M && id < I)) { M = p.x; I = id; }
  }
  ids[r] = I == 0x7fffffff ? 0 : I;
}

// Vocab-parallel argmax merge over peer memory (replaces an all-gather + merge): one CTA
// pushes this rank's (max, id) pairs [R] into slot [rank] of every peer's receive area and
// publishes the epoch; it then waits (bounded) for the W ranks and merges their pairs in
// rank order, ties to the smaller id.  Every rank computes the same ids.
__global__ void argmax_merge_ar_kernel(const float2* __restrict__ mine, int R, int* __restrict__ ids, ArDesc ar) {
  pdl_entry();
  const unsigned long long epoch = ar_epoch(ar);
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    const float2 v = mine[r];
    for (int q = 0; q < ar.world; q++) reinterpret_cast<float2*>(ar_slot(ar, q, epoch, ar.rank))[r] = v;
  }
  ar_producer_arrive(ar, epoch);
  const bool ok = ar_consumer_wait(ar, epoch);
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    float M = -INFINITY; int I = 0x7fffffff;
    if (ok)
      for (int w = 0; w < ar.world; w++) {
        const float2 p = reinterpret_cast<const float2*>(ar_slot(ar, ar.rank, epoch, w))[r];
        const int id = __float_as_int(p.y);
        if (p.x > M || (p.x == M && id < I)) { M = p.x; I = id; }
      }
    ids[r] = I == 0x7fffffff ? 0 : I;
  }
  ar_consumer_done(ar);
}

}  // namespace moet

using namespace moet;

void argmax_merge_ar(torch::Tensor mv, torch::Tensor ids, torch::Tensor ar) {
  TORCH_CHECK(mv.scalar_type() == at::kFloat && mv.dim() == 2 && mv.size(1) == 2 && mv.is_contiguous(),
              "argmax_merge_ar: mv [R, 2] f32");
  const int R = mv.size(0);
  ArDesc d = ar_desc_from(ar);
  TORCH_CHECK(ids.numel() >= R && 2LL * R <= d.cap, "argmax_merge_ar: ids / slot size");
  if (R == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_k(argmax_merge_ar_kernel, 1, 256, 0, stream, (const float2*)mv.data_ptr(), R, ids.data_ptr<int>(), d);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void argmax_split(torch::Tensor logits, c10::optional<torch::Tensor> ids, c10::optional<torch::Tensor> lse,
                  c10::optional<torch::Tensor> status, torch::Tensor part, torch::Tensor counter,
                  c10::optional<torch::Tensor> mv, int64_t id_offset) {
  const int R = logits.size(0), V = logits.size(1);
  TORCH_CHECK(logits.stride(1) == 1, "argmax_split: inner stride 1");
  const int S = part.size(1);
  TORCH_CHECK(part.size(0) >= R && part.size(2) == 3 && counter.numel() >= R, "argmax_split: scratch shapes");
  if (R == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  dim3 grid(R, S);
  const int want = lse.has_value() && lse->defined();
  if (logits.scalar_type() == at::kFloat)
    launch_k(argmax_split_kernel<float>, grid, 256, 0, stream, logits.data_ptr<float>(), logits.stride(0), V, want,
        part.data_ptr<float>(), counter.data_ptr<int>(), (int*)opt_ptr(ids), (float*)opt_ptr(lse), (int*)opt_ptr(status),
        (float2*)opt_ptr(mv), (int)id_offset);
  else
    launch_k(argmax_split_kernel<__nv_bfloat16>, grid, 256, 0, stream, (const __nv_bfloat16*)logits.data_ptr(),
        logits.stride(0), V, want, part.data_ptr<float>(), counter.data_ptr<int>(), (int*)opt_ptr(ids),
        (float*)opt_ptr(lse), (int*)opt_ptr(status), (float2*)opt_ptr(mv), (int)id_offset);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void argmax_merge(torch::Tensor parts, torch::Tensor ids) {
  TORCH_CHECK(parts.scalar_type() == at::kFloat && parts.dim() == 3 && parts.size(2) == 2 && parts.is_contiguous(),
              "argmax_merge: parts [W, R, 2] f32");
  const int W = parts.size(0), R = parts.size(1);
  TORCH_CHECK(ids.numel() >= R, "argmax_merge: ids too small");
  if (R == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_k(argmax_merge_kernel, (R + 127) / 128, 128, 0, stream, (const float2*)parts.data_ptr(), W, R, ids.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void argmax_lse(torch::Tensor logits, torch::Tensor ids, c10::optional<torch::Tensor> lse,
                c10::optional<torch::Tensor> maxv, c10::optional<torch::Tensor> status) {
  const int R = logits.size(0), V = logits.size(1);
  TORCH_CHECK(logits.stride(1) == 1, "argmax_lse: inner stride 1");
  if (R == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (logits.scalar_type() == at::kFloat)
    launch_k(argmax_lse_kernel<float>, R, 1024, 0, stream, logits.data_ptr<float>(), logits.stride(0), V, ids.data_ptr<int>(),
                                                     (float*)opt_ptr(lse), (float*)opt_ptr(maxv), (int*)opt_ptr(status));
  else
    launch_k(argmax_lse_kernel<__nv_bfloat16>, R, 1024, 0, stream, (const __nv_bfloat16*)logits.data_ptr(), logits.stride(0), V,
                                                             ids.data_ptr<int>(), (float*)opt_ptr(lse), (float*)opt_ptr(maxv),
                                                             (int*)opt_ptr(status));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mtp_accept(torch::Tensor targets, torch::Tensor tokens, torch::Tensor out_tokens, torch::Tensor n_acc,
                c10::optional<torch::Tensor> active) {
  const int B = targets.size(0), kp1 = targets.size(1);
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_k(mtp_accept_kernel, (B + 127) / 128, 128, 0, stream, targets.data_ptr<int>(), tokens.data_ptr<int>(), B, kp1,
                                                         out_tokens.data_ptr<int>(), n_acc.data_ptr<int>(),
                                                         (const int*)opt_ptr(active));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mtp_finalize(torch::Tensor targets, torch::Tensor n_acc, torch::Tensor drafts, torch::Tensor tokens,
                  torch::Tensor seq_pos, c10::optional<torch::Tensor> active) {
  const int B = targets.size(0), kp1 = targets.size(1);
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_k(mtp_finalize_kernel, (B + 127) / 128, 128, 0, stream, targets.data_ptr<int>(), n_acc.data_ptr<int>(),
                                                           drafts.data_ptr<int>(), B, kp1, tokens.data_ptr<int>(),
                                                           seq_pos.data_ptr<int>(), (const int*)opt_ptr(active));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
