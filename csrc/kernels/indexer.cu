// Sparse-attention indexer (DeepSeek DSA "lightning indexer" semantics):
//   score[t, s] = sum_h w[t, h] * relu(q[t, h, :] . k[s, :])      s < pos[t] + 1
// then the top-k positions per query feed the sparse MLA decode
// (mla_decode with a selection list).
//
// indexer_logits: one CTA per (token, 64-key block of its sequence).  The 64
// keys (bf16, [blocks, 64, D] paged like the latent cache) and the token's
// H_i query rows go to shared memory; S = Q K^T runs on mma.sync bf16
// (m16n8k16, fp32 accumulate), ReLU and the head-weighted sum reduce it to 64
// scores.  Positions past the causal end get -inf.
//
// indexer_topk: one CTA per query row.  Radix select on order-preserving
// uint32 keys: four 8-bit digit passes with shared-memory histograms find the
// k-th largest key exactly; the output lists every position above it plus the
// lowest-index ties, in increasing position order (block scans, so the result
// is deterministic), padded with -1.
#include "common.cuh"
#include "torch_glue.h"

namespace moet {

constexpr int kIdxBS = 64;

template <int D>
__global__ void __launch_bounds__(128) indexer_logits_kernel(const __nv_bfloat16* __restrict__ q, int Hi,
                                                             const float* __restrict__ w,
                                                             const __nv_bfloat16* __restrict__ kc, int n_blocks,
                                                             const int* __restrict__ block_table, int bt_stride,
                                                             const int* __restrict__ seq_of_tok,
                                                             const int* __restrict__ pos_of_tok,
                                                             float* __restrict__ out, int out_stride,
                                                             int* __restrict__ status) {
  pdl_entry();
  constexpr int kP = D + 8;                       // padded smem row (bf16) -> conflict-free ldmatrix
  __shared__ __align__(16) __nv_bfloat16 ks[kIdxBS * kP];
  __shared__ __align__(16) __nv_bfloat16 qsm[64 * kP];
  __shared__ float wsm[64];
  __shared__ float part[4][kIdxBS];
  const int tok = blockIdx.x, tile = blockIdx.y;
  const int L = pos_of_tok[tok] + 1;
  float* orow = out + (size_t)tok * out_stride;
  if (tile * kIdxBS >= L) {                        // beyond the causal end: -inf
    for (int j = threadIdx.x; j < kIdxBS; j += blockDim.x)
      if (tile * kIdxBS + j < out_stride) orow[tile * kIdxBS + j] = -INFINITY;
    return;
  }
  int blk = block_table[(size_t)seq_of_tok[tok] * bt_stride + tile];
  if (blk < 0 || blk >= n_blocks) { set_status(status, kBadIndex); blk = 0; }
  const __nv_bfloat16* kb = kc + (size_t)blk * kIdxBS * D;
  for (int i = threadIdx.x; i < kIdxBS * D / 8; i += blockDim.x) {
    const int r = i / (D / 8), c = (i % (D / 8)) * 8;
    *reinterpret_cast<uint4*>(ks + r * kP + c) = *reinterpret_cast<const uint4*>(kb + (size_t)r * D + c);
  }
  const int HiP = (Hi + 15) / 16 * 16;
  for (int i = threadIdx.x; i < HiP * D / 8; i += blockDim.x) {
    const int r = i / (D / 8), c = (i % (D / 8)) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < Hi) v = *reinterpret_cast<const uint4*>(q + ((size_t)tok * Hi + r) * D + c);
    *reinterpret_cast<uint4*>(qsm + r * kP + c) = v;
  }
  for (int i = threadIdx.x; i < HiP; i += blockDim.x) wsm[i] = i < Hi ? w[(size_t)tok * Hi + i] : 0.f;
  __syncthreads();
  // warp w: keys [16w, 16w+16) (two n8 tiles), all head tiles
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  float sc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};       // [n8 tile][column pair] head-weighted relu sums
  for (int m0 = 0; m0 < HiP; m0 += 16) {
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < D / 16; kk++) {
      uint32_t a[4];
      ldmatrix_x4(a, qsm + (m0 + (lane & 15)) * kP + kk * 16 + (lane >> 4) * 8);
#pragma unroll
      for (int nt = 0; nt < 2; nt++) {
        uint32_t b[2];
        ldmatrix_x2(b, ks + (warp * 16 + nt * 8 + (lane & 7)) * kP + kk * 16 + ((lane >> 3) & 1) * 8);
        mma_bf16_16816(acc[nt], a, b[0], b[1]);
      }
    }
    // rows g and g+8 are heads m0+g, m0+g+8; columns 2t, 2t+1 are keys
#pragma unroll
    for (int nt = 0; nt < 2; nt++) {
      sc[nt][0] += wsm[m0 + g] * fmaxf(acc[nt][0], 0.f) + wsm[m0 + g + 8] * fmaxf(acc[nt][2], 0.f);
      sc[nt][1] += wsm[m0 + g] * fmaxf(acc[nt][1], 0.f) + wsm[m0 + g + 8] * fmaxf(acc[nt][3], 0.f);
    }
  }
  // sum over the 8 row groups (lanes with equal t)
#pragma unroll
  for (int nt = 0; nt < 2; nt++)
#pragma unroll
    for (int c = 0; c < 2; c++) {
      float v = sc[nt][c];
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      if (g == 0) part[0][warp * 16 + nt * 8 + 2 * t + c] = v;
    }
  __syncthreads();
  for (int j = threadIdx.x; j < kIdxBS; j += blockDim.x) {
    const int pos = tile * kIdxBS + j;
    if (pos < out_stride) orow[pos] = pos < L ? part[0][j] : -INFINITY;
  }
}

MOET_DEVICE uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);   // larger float -> larger key; -inf smallest finite order
}

constexpr int kTopkThreads = 1024;

__global__ void __launch_bounds__(kTopkThreads) indexer_topk_kernel(const float* __restrict__ scores, int S,
                                                                   int stride, int k, int* __restrict__ out) {
  pdl_entry();
  __shared__ unsigned hist[256];
  __shared__ unsigned prefix_s, remain_s;
  __shared__ int scan[kTopkThreads];
  const float* row = scores + (size_t)blockIdx.x * stride;
  int* orow = out + (size_t)blockIdx.x * k;
  // count finite candidates: -inf entries never qualify
  unsigned prefix = 0, mask = 0, remain = k;
  for (int d = 3; d >= 0; d--) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < S; i += blockDim.x) {
      const float f = row[i];
      if (f == -INFINITY) continue;
      const uint32_t key = order_key(f);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> (8 * d)) & 0xFF], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned cum = 0;
      int b = 255;
      for (; b >= 0; b--) {
        if (cum + hist[b] >= remain) break;
        cum += hist[b];
      }
      if (b < 0) {   // fewer than k finite candidates: take all of them
        prefix_s = 0xFFFFFFFFu; remain_s = 0;
      } else {
        prefix_s = prefix | ((unsigned)b << (8 * d));
        remain_s = remain - cum;
      }
    }
    __syncthreads();
    if (prefix_s == 0xFFFFFFFFu) { prefix = 0; mask = 0; remain = 0; break; }
    prefix = prefix_s; remain = remain_s; mask |= 0xFFu << (8 * d);
    __syncthreads();
  }
  // thr = k-th largest key (exact); take every key > thr, and the first `remain` keys == thr
  const bool all = (mask == 0);
  const uint32_t thr = prefix;
  const int per = (S + blockDim.x - 1) / blockDim.x;
  const int lo = threadIdx.x * per, hi = min(S, lo + per);
  int n_gt = 0, n_eq = 0;
  for (int i = lo; i < hi; i++) {
    const float f = row[i];
    if (f == -INFINITY) continue;
    const uint32_t key = order_key(f);
    if (all || key > thr) n_gt++;
    else if (key == thr) n_eq++;
  }
  // exclusive scans of n_eq (to pick the first ties) then of the selected counts
  scan[threadIdx.x] = n_eq;
  __syncthreads();
  for (int off = 1; off < blockDim.x; off <<= 1) {
    const int v = threadIdx.x >= off ? scan[threadIdx.x - off] : 0;
    __syncthreads();
    scan[threadIdx.x] += v;
    __syncthreads();
  }
  const int eq_before = scan[threadIdx.x] - n_eq;
  const int take_eq = all ? 0 : max(0, min(n_eq, (int)remain - eq_before));
  const int mine = n_gt + take_eq;
  __syncthreads();
  scan[threadIdx.x] = mine;
  __syncthreads();
  for (int off = 1; off < blockDim.x; off <<= 1) {
    const int v = threadIdx.x >= off ? scan[threadIdx.x - off] : 0;
    __syncthreads();
    scan[threadIdx.x] += v;
    __syncthreads();
  }
  int o = scan[threadIdx.x] - mine;
  const int total = scan[blockDim.x - 1];
  int eq_left = take_eq;
  for (int i = lo; i < hi; i++) {
    const float f = row[i];
    if (f == -INFINITY) continue;
    const uint32_t key = order_key(f);
    if (all || key > thr) orow[o++] = i;
    else if (key == thr && eq_left > 0) { orow[o++] = i; eq_left--; }
  }
  for (int i = total + threadIdx.x; i < k; i += blockDim.x) orow[i] = -1;
}

// Indexer key cache insert: cache[slot[t]] = k[t] (bf16 rows of D); slot < 0 skips.
__global__ void idx_k_write_kernel(const __nv_bfloat16* __restrict__ k, int D, const long long* __restrict__ slot,
                                   long long n_slots, __nv_bfloat16* __restrict__ cache, int* __restrict__ status) {
  pdl_entry();
  const long long s = slot[blockIdx.x];
  if (s < 0) return;
  if (s >= n_slots) { if (threadIdx.x == 0) set_status(status, kBadIndex); return; }
  for (int i = threadIdx.x * 8; i < D; i += blockDim.x * 8)
    *reinterpret_cast<uint4*>(cache + s * D + i) = *reinterpret_cast<const uint4*>(k + (size_t)blockIdx.x * D + i);
}

}  // namespace moet

using namespace moet;

void idx_k_write(torch::Tensor k, torch::Tensor slot, torch::Tensor cache, torch::Tensor status) {
  const int T = k.size(0), D = k.size(1);
  TORCH_CHECK(k.scalar_type() == at::kBFloat16 && k.is_contiguous() && D % 8 == 0 && cache.size(-1) == D &&
              slot.scalar_type() == at::kLong, "idx_k_write: k [T, D] bf16, slot int64");
  if (T == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_k(idx_k_write_kernel, T, 32, 0, stream, (const __nv_bfloat16*)k.data_ptr(), D,
           (const long long*)slot.data_ptr<int64_t>(), (long long)(cache.numel() / D),
           (__nv_bfloat16*)cache.data_ptr(), status.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void indexer_logits(torch::Tensor q, torch::Tensor w, torch::Tensor k_cache, torch::Tensor block_table,
                    torch::Tensor seq_of_tok, torch::Tensor pos_of_tok, torch::Tensor out, torch::Tensor status) {
  const int T = q.size(0), Hi = q.size(1), D = q.size(2);
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && Hi <= 64, "indexer_logits: q [T, <=64, D] bf16");
  TORCH_CHECK(k_cache.scalar_type() == at::kBFloat16 && k_cache.size(1) == kIdxBS && k_cache.size(2) == D &&
              k_cache.is_contiguous(), "indexer_logits: k cache [blocks, 64, D] bf16");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && w.size(0) == T && w.size(1) == Hi, "indexer_logits: w");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.stride(1) == 1 && out.size(0) == T, "indexer_logits: out [T, S]");
  if (T == 0) return;
  const int S = out.size(1);
  auto stream = at::cuda::getCurrentCUDAStream();
  dim3 grid(T, (S + kIdxBS - 1) / kIdxBS);
  TORCH_CHECK(D == 128, "indexer_logits: head dim 128");
  launch_k(indexer_logits_kernel<128>, grid, 128, 0, stream, (const __nv_bfloat16*)q.data_ptr(), Hi,
           w.data_ptr<float>(), (const __nv_bfloat16*)k_cache.data_ptr(), (int)k_cache.size(0),
           block_table.data_ptr<int>(), (int)block_table.stride(0), seq_of_tok.data_ptr<int>(),
           pos_of_tok.data_ptr<int>(), out.data_ptr<float>(), (int)out.stride(0), status.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void indexer_topk(torch::Tensor scores, int64_t k, torch::Tensor out) {
  TORCH_CHECK(scores.scalar_type() == at::kFloat && scores.stride(1) == 1, "indexer_topk: scores [T, S] f32");
  TORCH_CHECK(out.scalar_type() == at::kInt && out.is_contiguous() && out.size(0) == scores.size(0) && out.size(1) == k,
              "indexer_topk: out [T, k] int32");
  const int T = scores.size(0), S = scores.size(1);
  if (T == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_k(indexer_topk_kernel, T, kTopkThreads, 0, stream, scores.data_ptr<float>(), S, (int)scores.stride(0),
           (int)k, out.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
