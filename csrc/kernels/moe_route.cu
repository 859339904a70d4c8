// Router top-k and the expert pair-list builder.
//
// Router (one warp per token): sigmoid scores with a selection bias
// ("noaux" correction, DeepSeek-V3/V4 style) and optional group-limited
// selection, or softmax scores; top-k by repeated warp argmax with ties
// broken toward the lower expert id; weights renormalised and scaled.
//
// Pair-list builder (one CTA): groups the T*k routings by expert and cuts
// each expert's rows into "pairs" of at most MB rows -- the work items of
// the expert GEMV/GEMM (reference: moe_align_block_size + the Triton desc
// builders, P:6198-6254, P:7389).  Everything stays on the device so a
// captured CUDA graph replays any routing.  Numerics do not depend on the
// order of rows inside an expert (each output column is independent).
#include "common.cuh"
#include "ep_a2a.cuh"
#include "torch_glue.h"

namespace moet {

constexpr int kMaxE = 512;

// Top-k of one token's router logits (one warp): sigmoid + selection bias (or
// softmax), optional group limit, renormalised and scaled weights.
// PER = values per lane (E <= 32 * PER); the k selection rounds cost O(PER).
template <int PER>
__device__ __forceinline__ void topk_token_t(const float* __restrict__ logits, const float* __restrict__ bias,
                                             int warp, int E, int k, int sigmoid, int n_group, int topk_group,
                                             int norm, float scaling, int* __restrict__ ids, float* __restrict__ wts) {
  const int lane = threadIdx.x & 31;
  float score[PER], sel[PER];
  const int per = (E + 31) / 32;
  const float* lg = logits + (size_t)warp * E;
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; i++) {
    const int e = lane + 32 * i;
    float v = (i < per && e < E) ? lg[e] : -INFINITY;
    score[i] = v;
    mx = fmaxf(mx, v);
  }
  if (sigmoid) {
#pragma unroll
    for (int i = 0; i < PER; i++) {
      const int e = lane + 32 * i;
      if (i < per && e < E) {
        score[i] = 1.f / (1.f + __expf(-score[i]));
        sel[i] = score[i] + (bias ? bias[e] : 0.f);
      } else { score[i] = 0.f; sel[i] = -INFINITY; }
    }
  } else {
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < PER; i++) {
      const int e = lane + 32 * i;
      float v = (i < per && e < E) ? __expf(score[i] - mx) : 0.f;
      score[i] = v; sum += v;
    }
    sum = warp_sum(sum);
#pragma unroll
    for (int i = 0; i < PER; i++) {
      const int e = lane + 32 * i;
      score[i] /= sum;
      sel[i] = (i < per && e < E) ? score[i] : -INFINITY;
    }
  }
  if (n_group > 1 && topk_group < n_group) {
    // group score = sum of the two best selection scores in the group; keep topk_group groups
    const int gsize = E / n_group;
    __shared__ float gscore_s[16][64];
    float* gscore = gscore_s[(threadIdx.x >> 5) & 15];
    __syncwarp();
    // Compute group scores cooperatively: each lane owns experts lane+32i.
    for (int gi = 0; gi < n_group; gi++) {
      float b1 = -INFINITY, b2 = -INFINITY;
#pragma unroll
      for (int i = 0; i < PER; i++) {
        const int e = lane + 32 * i;
        if (i < per && e < E && e / gsize == gi) {
          float v = sel[i];
          if (v > b1) { b2 = b1; b1 = v; } else if (v > b2) b2 = v;
        }
      }
      // warp-merge top-2
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        float o1 = __shfl_xor_sync(0xffffffffu, b1, o), o2 = __shfl_xor_sync(0xffffffffu, b2, o);
        float n1 = fmaxf(b1, o1);
        float n2 = fmaxf(fminf(b1, o1), fmaxf(b2, o2));
        b1 = n1; b2 = n2;
      }
      if (lane == 0) gscore[gi] = b1 + (gsize > 1 ? b2 : 0.f);
    }
    __syncwarp();
    // choose topk_group groups (ties -> lower group id)
    unsigned long long keep = 0;
    for (int r = 0; r < topk_group; r++) {
      int best = -1; float bv = -INFINITY;
      for (int gi = 0; gi < n_group; gi++)
        if (!((keep >> gi) & 1ull) && (best < 0 || gscore[gi] > bv)) { best = gi; bv = gscore[gi]; }
      keep |= 1ull << best;
    }
#pragma unroll
    for (int i = 0; i < PER; i++) {
      const int e = lane + 32 * i;
      if (i < per && e < E && !((keep >> (e / gsize)) & 1ull)) sel[i] = -INFINITY;
    }
  }
  float wsum = 0.f;
  float myw = 0.f; int myid = 0;
  for (int r = 0; r < k; r++) {
    float bv = -INFINITY; int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; i++) {
      const int e = lane + 32 * i;
      if (i < per && e < E && (sel[i] > bv || (sel[i] == bv && e < bi))) { bv = sel[i]; bi = e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    // owner lane reads the raw score and removes the expert from selection
    float w = 0.f;
#pragma unroll
    for (int i = 0; i < PER; i++) {
      const int e = lane + 32 * i;
      if (e == bi) { w = score[i]; sel[i] = -INFINITY; }
    }
    w = __shfl_sync(0xffffffffu, w, bi & 31);
    wsum += w;
    if (lane == r) { myw = w; myid = bi; }
  }
  if (lane < k) {
    float w = myw;
    if (norm) w = w / (wsum + 1e-20f);
    ids[(size_t)warp * k + lane] = myid;
    wts[(size_t)warp * k + lane] = w * scaling;
  }
}

__device__ __forceinline__ void topk_token(const float* __restrict__ logits, const float* __restrict__ bias,
                                           int warp, int E, int k, int sigmoid, int n_group, int topk_group,
                                           int norm, float scaling, int* __restrict__ ids, float* __restrict__ wts) {
  if (E <= 128)
    topk_token_t<4>(logits, bias, warp, E, k, sigmoid, n_group, topk_group, norm, scaling, ids, wts);
  else if (E <= 256)
    topk_token_t<8>(logits, bias, warp, E, k, sigmoid, n_group, topk_group, norm, scaling, ids, wts);
  else
    topk_token_t<kMaxE / 32>(logits, bias, warp, E, k, sigmoid, n_group, topk_group, norm, scaling, ids, wts);
}

__global__ void router_topk_kernel(const float* __restrict__ logits, const float* __restrict__ bias,
                                   int T, int E, int k, int sigmoid, int n_group, int topk_group,
                                   int norm, float scaling, int* __restrict__ ids, float* __restrict__ wts) {
  pdl_entry();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (warp >= T) return;
  topk_token(logits, bias, warp, E, k, sigmoid, n_group, topk_group, norm, scaling, ids, wts);
}

// ---------------------------------------------------------------------------
// Router logits: logits[t, e] = x[t, :] . W[e, :] with bf16 x and W, fp32 sums.
// One warp per expert, 16-byte vector loads, 8 tokens per pass.
__global__ void router_logits_kernel(const __nv_bfloat16* __restrict__ x, int T, int H,
                                     const __nv_bfloat16* __restrict__ w, int E, float* __restrict__ out) {
  {  // router weights are immutable: prefetch this CTA's experts' rows before waiting on x
    const int e0 = blockIdx.x * (blockDim.x >> 5), ne = min((int)(blockDim.x >> 5), E - e0);
    const char* wb = reinterpret_cast<const char*>(w + (size_t)e0 * H);
    for (int i = threadIdx.x; i < ne * H * 2 / 128; i += blockDim.x) prefetch_l2(wb + (size_t)i * 128);
  }
  pdl_entry();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * (blockDim.x >> 5) + warp;
  if (e >= E) return;
  const __nv_bfloat16* wr = w + (size_t)e * H;
  for (int t0 = 0; t0 < T; t0 += 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int k = lane * 8; k < H; k += 256) {
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(wr + k));
      const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wv);
      float wf[8];
#pragma unroll
      for (int i = 0; i < 4; i++) { const float2 f = __bfloat1622float2(w2[i]); wf[2 * i] = f.x; wf[2 * i + 1] = f.y; }
#pragma unroll
      for (int j = 0; j < 8; j++) {
        if (t0 + j >= T) break;
        const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + (size_t)(t0 + j) * H + k));
        const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xv);
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float2 f = __bfloat1622float2(x2[i]);
          acc[j] = fmaf(f.x, wf[2 * i], fmaf(f.y, wf[2 * i + 1], acc[j]));
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const float v = warp_sum(acc[j]);
      if (lane == 0 && t0 + j < T) out[(size_t)(t0 + j) * E + e] = v;
    }
  }
}

// Prefill router logits on the tensor cores: out[T, E] (f32) = x[T, H] (bf16) . w[E, H]^T (bf16),
// fp32 accumulation -- the same operands and precision as the decode router above.  A CTA
// computes a 64-token x 64-expert tile; 64-k slices of both operands are staged with
// cp.async (double-buffered, rows padded by 16 bytes so ldmatrix is conflict-free) and
// consumed by bf16 m16n8k16 MMAs, one 16-token strip per warp.
__global__ void __launch_bounds__(128) router_logits_mma_kernel(const __nv_bfloat16* __restrict__ x, int T, int H,
                                                                const __nv_bfloat16* __restrict__ w, int E,
                                                                float* __restrict__ out, float* __restrict__ part,
                                                                int* __restrict__ cnt, int kslice) {
  constexpr int BT = 64, BE = 64, BK = 64, LD = BK + 8;
  __shared__ __align__(16) __nv_bfloat16 sx[2][BT * LD];
  __shared__ __align__(16) __nv_bfloat16 sw[2][BE * LD];
  const int t0 = blockIdx.x * BT, e0 = blockIdx.y * BE;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  auto load = [&](int buf, int k0, bool act) {
    for (int i = tid; i < BT * BK / 8; i += 128) {
      const int r = i >> 3, c = (i & 7) * 8;
      const uint32_t dw = (uint32_t)__cvta_generic_to_shared(&sw[buf][r * LD + c]);
      const __nv_bfloat16* srcw = w + (size_t)(e0 + r) * H + k0 + c;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dw), "l"(srcw) : "memory");
      if (act) {
        const bool ok = t0 + r < T;
        const uint32_t dx = (uint32_t)__cvta_generic_to_shared(&sx[buf][r * LD + c]);
        const __nv_bfloat16* srcx = ok ? x + (size_t)(t0 + r) * H + k0 + c : x;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dx), "l"(srcx), "r"(ok ? 16 : 0) : "memory");
      }
    }
  };
  // K slice of this CTA (grid.z): chunks [kc0, kc0 + nk) of 64
  const int kc0 = blockIdx.z * (kslice / BK), nk = min(kslice, H - blockIdx.z * kslice) / BK;
  // router weights are immutable: their first slice may load before the previous kernel ends
  load(0, kc0 * BK, false);
  pdl_entry();
  load(0, kc0 * BK, true);
  asm volatile("cp.async.commit_group;" ::: "memory");
  float acc[8][4];
#pragma unroll
  for (int n = 0; n < 8; n++) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  for (int kc = 0; kc < nk; kc++) {
    if (kc + 1 < nk) load((kc + 1) & 1, (kc0 + kc + 1) * BK, true);
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncthreads();
    const __nv_bfloat16* ax = sx[kc & 1];
    const __nv_bfloat16* bw = sw[kc & 1];
#pragma unroll
    for (int kk = 0; kk < BK / 16; kk++) {
      uint32_t a[4];
      ldmatrix_x4(a, ax + (warp * 16 + (lane & 15)) * LD + kk * 16 + (lane >> 4) * 8);
#pragma unroll
      for (int n = 0; n < 8; n++) {
        uint32_t b[2];
        ldmatrix_x2(b, bw + (n * 8 + (lane & 7)) * LD + kk * 16 + ((lane >> 3) & 1) * 8);
        mma_bf16_16816(acc[n], a, b[0], b[1]);
      }
    }
    __syncthreads();
  }
  const int r0 = t0 + warp * 16 + g;
  const int ks = gridDim.z;
  // one slice: straight to out; several: partials to part[z], and the tile's last CTA (arrival
  // counter, self-resetting) adds them in slice order -- the same sum on every run and rank
  float* dst = ks == 1 ? out : part + (size_t)blockIdx.z * T * E;
#pragma unroll
  for (int n = 0; n < 8; n++) {
    const int col = e0 + n * 8 + 2 * t;
    if (r0 < T) *reinterpret_cast<float2*>(dst + (size_t)r0 * E + col) = make_float2(acc[n][0], acc[n][1]);
    if (r0 + 8 < T) *reinterpret_cast<float2*>(dst + (size_t)(r0 + 8) * E + col) = make_float2(acc[n][2], acc[n][3]);
  }
  if (ks == 1) return;
  __shared__ int last;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    int* c = cnt + blockIdx.y * gridDim.x + blockIdx.x;
    last = atomicAdd(c, 1) == ks - 1;
    if (last) *c = 0;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int i = tid; i < BT * BE / 4; i += 128) {
    const int r = t0 + (i * 4) / BE, col = e0 + (i * 4) % BE;
    if (r >= T) continue;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int z = 0; z < ks; z++) {
      const float4 u = __ldcg(reinterpret_cast<const float4*>(part + ((size_t)z * T + r) * E + col));
      v.x += u.x; v.y += u.y; v.z += u.z; v.w += u.w;
    }
    *reinterpret_cast<float4*>(out + (size_t)r * E + col) = v;
  }
}

// ---------------------------------------------------------------------------
// Pair-list builder.  outputs:
//   sorted_tok[R]   token of each expert-sorted row
//   pos_of[R]       routing r (= t*k + j) -> sorted row
//   pairs[P] int4   {expert, first sorted row, n rows (<= MB), 0}
//   n_pairs[1]
// Block-wide body (blockDim.x >= E, a multiple of 32).
__device__ __forceinline__ void build_pairs_block(const int* __restrict__ topk_ids, int R, int k, int E, int MB,
                                                  int* __restrict__ rank_scratch, int* __restrict__ sorted_tok,
                                                  int* __restrict__ pos_of, int4* __restrict__ pairs,
                                                  int* __restrict__ n_pairs, int* __restrict__ status,
                                                  int pad, int* __restrict__ n_rows, int e_lo = 0, int ep = 0) {
  // ep != 0: expert parallelism -- this rank owns experts [e_lo, e_lo + E); routings to other
  // experts are skipped (pos_of = -1, the combine ignores them); pairs carry local expert ids
  __shared__ int cnt[kMaxE];
  __shared__ int start[kMaxE];
  __shared__ int pstart[kMaxE];
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    int e = topk_ids[r] - e_lo;
    if (e < 0 || e >= E) {
      if (ep) { rank_scratch[r] = -1; continue; }
      set_status(status, kBadIndex); e = 0;
    }
    rank_scratch[r] = atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  // exclusive prefix sums of the row counts and pair counts (block scan, E <= 512)
  {
    __shared__ int wtot_c[32], wtot_p[32];
    const int e = threadIdx.x, lane = e & 31, w = e >> 5;
    const int c0 = e < E ? cnt[e] : 0, pc = (c0 + MB - 1) / MB;
    const int c = pad ? pc * MB : c0;          // padded: every segment starts at a multiple of MB
    int ic = c, ip = pc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int a = __shfl_up_sync(0xffffffffu, ic, o), b = __shfl_up_sync(0xffffffffu, ip, o);
      if (lane >= o) { ic += a; ip += b; }
    }
    if (lane == 31) { wtot_c[w] = ic; wtot_p[w] = ip; }
    __syncthreads();
    if (w == 0) {
      const int nw = blockDim.x >> 5;
      int tc = lane < nw ? wtot_c[lane] : 0, tp = lane < nw ? wtot_p[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, tc, o), b = __shfl_up_sync(0xffffffffu, tp, o);
        if (lane >= o) { tc += a; tp += b; }
      }
      if (lane < nw) { wtot_c[lane] = tc; wtot_p[lane] = tp; }  // inclusive over warps
    }
    __syncthreads();
    const int offc = w ? wtot_c[w - 1] : 0, offp = w ? wtot_p[w - 1] : 0;
    if (e < E) { start[e] = offc + ic - c; pstart[e] = offp + ip - pc; }
    if (e == E - 1) { *n_pairs = offp + ip; if (n_rows) *n_rows = offc + ic; }
  }
  __syncthreads();
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    int e = topk_ids[r] - e_lo;
    if (e < 0 || e >= E) {
      if (ep) { pos_of[r] = -1; continue; }
      e = 0;
    }
    const int pos = start[e] + rank_scratch[r];
    sorted_tok[pos] = r / k;
    pos_of[r] = pos;
  }
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int c = cnt[e];
    for (int i = 0; i * MB < c; i++)
      pairs[pstart[e] + i] = make_int4(e, start[e] + i * MB, min(MB, c - i * MB), 0);
    if (pad)   // padding rows of the segment map to no token
      for (int i = c; i < (c + MB - 1) / MB * MB; i++) sorted_tok[start[e] + i] = -1;
  }
}

__global__ void build_pairs_kernel(const int* __restrict__ topk_ids, int R, int k, int E, int MB,
                                   int* __restrict__ rank_scratch, int* __restrict__ sorted_tok,
                                   int* __restrict__ pos_of, int4* __restrict__ pairs,
                                   int* __restrict__ n_pairs, int* __restrict__ status,
                                   int pad = 0, int* __restrict__ n_rows = nullptr, int e_lo = 0, int ep = 0) {
  pdl_entry();
  build_pairs_block(topk_ids, R, k, E, MB, rank_scratch, sorted_tok, pos_of, pairs, n_pairs, status, pad, n_rows,
                    e_lo, ep);
}

// Expert parallelism, owner side (protocol in ep_a2a.cuh).  One CTA of 1024 threads:
// bounded wait for every source's dispatch flag, then the expert pair list of the rows
// received -- ids[r] = local expert id of received row r = src * cap + i, -1 for empty
// slots (skipped) -- with sorted row -> received row index in sorted_tok.
__global__ void __launch_bounds__(1024) ep_recv_pairs_kernel(EpDesc d, int MB, int* __restrict__ ids,
                                                             int* __restrict__ rank_scratch,
                                                             int* __restrict__ sorted_tok, int* __restrict__ pos_of,
                                                             int4* __restrict__ pairs, int* __restrict__ n_pairs,
                                                             int* __restrict__ n_rows) {
  pdl_entry();
  const unsigned long long epoch = ep_epoch(d);
  const bool ok = ep_wait(d, epoch, 0);
  const int R = d.world * d.cap;
  const int* nrows = ep_nrows(d, d.rank);
  const int* meta = ep_meta(d, d.rank);
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    const int src = r / d.cap, i = r - src * d.cap;
    ids[r] = ok && i < nrows[src] ? meta[r] : -1;
  }
  __syncthreads();
  build_pairs_block(ids, R, 1, d.E_loc, MB, rank_scratch, sorted_tok, pos_of, pairs, n_pairs, d.status, 0, n_rows,
                    0, 1);
}

// Decode routing in one launch: every CTA computes the router logits of 4
// experts for all T tokens (4 warps per expert, each over a quarter of H;
// bf16 x and W, fp32 sums; the weight rows are loaded before the dependency
// wait); the last CTA to finish (arrival counter, self-resetting) runs the
// top-k of every token and builds the expert pair list.
constexpr int kRouteWarps = 16;
constexpr int kRouteExperts = 4;
__global__ void __launch_bounds__(kRouteWarps * 32) moe_route_fused_kernel(
    const __nv_bfloat16* __restrict__ x, int T, int H, const __nv_bfloat16* __restrict__ w, int E,
    float* __restrict__ logits, const float* __restrict__ bias, int k, int sigmoid, int n_group, int topk_group,
    int norm, float scaling, int* __restrict__ ids, float* __restrict__ wts, int MB,
    int* __restrict__ rank_scratch, int* __restrict__ sorted_tok, int* __restrict__ pos_of,
    int4* __restrict__ pairs, int* __restrict__ n_pairs, int* __restrict__ counter, int* __restrict__ status,
    int e_lo, int E_local, int ep) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int el = warp >> 2, qh = warp & 3;
  const int e = blockIdx.x * kRouteExperts + el;
  const int Hq = H >> 2, h0 = qh * Hq;
  constexpr int kPre = 8;
  const int nvec = Hq / 256;      // 16-byte vectors per lane in this quarter
  const __nv_bfloat16* wr = w + (size_t)min(e, E - 1) * H + h0;
  uint4 wv[kPre];
#pragma unroll
  for (int u = 0; u < kPre; u++)
    if (u < nvec) wv[u] = __ldg(reinterpret_cast<const uint4*>(wr + u * 256 + lane * 8));
  pdl_entry();
  extern __shared__ __align__(16) uint8_t route_smem[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(route_smem);   // [4][H]
  __shared__ float qpart[kRouteWarps][4];
  for (int t0 = 0; t0 < T; t0 += 4) {
    const int nt = min(4, T - t0);
    __syncthreads();
    for (int i = threadIdx.x; i < nt * H / 8; i += blockDim.x)
      reinterpret_cast<uint4*>(xs)[i] = __ldg(reinterpret_cast<const uint4*>(x + (size_t)t0 * H) + i);
    __syncthreads();
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int u0 = 0; u0 < nvec; u0 += kPre) {
#pragma unroll
      for (int u = 0; u < kPre; u++) {
        if (u0 + u >= nvec) break;
        const uint4 wq = u0 == 0 ? wv[u] : __ldg(reinterpret_cast<const uint4*>(wr + (u0 + u) * 256 + lane * 8));
        const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wq);
#pragma unroll
        for (int j = 0; j < 4; j++) {
          if (j < nt) {
            const uint4 xv = *reinterpret_cast<const uint4*>(xs + (size_t)j * H + h0 + (u0 + u) * 256 + lane * 8);
            const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xv);
#pragma unroll
            for (int i = 0; i < 4; i++) {
              const float2 a = __bfloat1622float2(x2[i]), b = __bfloat1622float2(w2[i]);
              acc[j] = fmaf(a.x, b.x, fmaf(a.y, b.y, acc[j]));
            }
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float v = warp_sum(acc[j]);
      if (lane == 0) qpart[warp][j] = v;
    }
    __syncthreads();
    if (threadIdx.x < kRouteExperts * 4) {      // (expert, token) -> sum of the 4 quarters in fixed order
      const int ee = threadIdx.x >> 2, j = threadIdx.x & 3, eg = blockIdx.x * kRouteExperts + ee;
      if (eg < E && j < nt)
        logits[(size_t)(t0 + j) * E + eg] = ((qpart[ee * 4][j] + qpart[ee * 4 + 1][j]) + qpart[ee * 4 + 2][j]) +
                                            qpart[ee * 4 + 3][j];
    }
  }
  __shared__ int last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(counter, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int t = warp; t < T; t += kRouteWarps)
    topk_token(logits, bias, t, E, k, sigmoid, n_group, topk_group, norm, scaling, ids, wts);
  __syncthreads();
  __threadfence_block();
  build_pairs_block(ids, T * k, k, ep ? E_local : E, MB, rank_scratch, sorted_tok, pos_of, pairs, n_pairs, status,
                    0, nullptr, e_lo, ep);
  if (threadIdx.x == 0) *counter = 0;
}

}  // namespace moet

using namespace moet;

void router_topk(torch::Tensor logits, c10::optional<torch::Tensor> bias, int64_t k, bool sigmoid,
                 int64_t n_group, int64_t topk_group, bool norm, double scaling, torch::Tensor ids,
                 torch::Tensor wts) {
  const int T = logits.size(0), E = logits.size(1);
  TORCH_CHECK(E <= kMaxE && k <= 32, "router_topk: E <= 512, k <= 32");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.is_contiguous(), "logits f32 contiguous");
  TORCH_CHECK(n_group <= 64, "router_topk: n_group <= 64");
  if (T == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  const int warps = 8;
  launch_k(router_topk_kernel, (T + warps - 1) / warps, warps * 32, 0, stream, 
      logits.data_ptr<float>(), bias.has_value() && bias->defined() ? bias->data_ptr<float>() : nullptr,
      T, E, (int)k, sigmoid ? 1 : 0, (int)n_group, (int)topk_group, norm ? 1 : 0, (float)scaling,
      ids.data_ptr<int>(), wts.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// dst[r] = src[idx[r]] (rows of e4m3 + their per-64 scales); idx < 0 -> zeros; rows >= *n_rows untouched.
__global__ void gather_rows_kernel(const uint8_t* __restrict__ src_q, const uint8_t* __restrict__ src_s, int K,
                                   long long src_stride, const int* __restrict__ idx, const int* __restrict__ n_rows,
                                   uint8_t* __restrict__ dst_q, uint8_t* __restrict__ dst_s, long long dst_stride) {
  pdl_entry();
  const int r = blockIdx.x;
  if (r >= *n_rows) return;
  const int i = idx[r];
  const int nv = K / 16;
  for (int c = threadIdx.x; c < nv; c += blockDim.x) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (i >= 0) v = __ldg(reinterpret_cast<const uint4*>(src_q + (size_t)i * src_stride) + c);
    reinterpret_cast<uint4*>(dst_q + (size_t)r * dst_stride)[c] = v;
  }
  for (int c = threadIdx.x; c < K / 64; c += blockDim.x)
    dst_s[(size_t)r * (K / 64) + c] = i >= 0 ? src_s[(size_t)i * (K / 64) + c] : 0;
}

void gather_rows(torch::Tensor src_q, torch::Tensor src_s, torch::Tensor idx, torch::Tensor n_rows, torch::Tensor dst_q,
                 torch::Tensor dst_s) {
  const int K = src_q.size(1), R = idx.size(0);
  TORCH_CHECK(K % 64 == 0 && src_q.stride(0) % 16 == 0 && dst_q.stride(0) % 16 == 0, "gather_rows: alignment");
  TORCH_CHECK(dst_q.size(0) >= R && dst_s.size(0) >= R, "gather_rows: destination too small");
  if (R == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_k(gather_rows_kernel, R, 128, 0, stream, (const uint8_t*)src_q.data_ptr(), (const uint8_t*)src_s.data_ptr(), K,
                                            src_q.stride(0), idx.data_ptr<int>(), n_rows.data_ptr<int>(),
                                            (uint8_t*)dst_q.data_ptr(), (uint8_t*)dst_s.data_ptr(), dst_q.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void moe_route_fused(torch::Tensor x, torch::Tensor w, torch::Tensor logits, c10::optional<torch::Tensor> bias,
                     int64_t k, bool sigmoid, int64_t n_group, int64_t topk_group, bool norm, double scaling,
                     torch::Tensor ids, torch::Tensor wts, int64_t MB, torch::Tensor rank_scratch,
                     torch::Tensor sorted_tok, torch::Tensor pos_of, torch::Tensor pairs, torch::Tensor n_pairs,
                     torch::Tensor counter, torch::Tensor status, int64_t e_lo, int64_t E_local) {
  const int T = x.size(0), H = x.size(1), E = w.size(0);
  const int ep = E_local > 0 ? 1 : 0;
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && x.is_contiguous() &&
              w.is_contiguous() && H % 1024 == 0, "moe_route_fused: bf16 contiguous, H % 1024 == 0");
  TORCH_CHECK(E <= kRouteWarps * 32 && k <= 32 && n_group <= 64, "moe_route_fused: E <= 512, k <= 32");
  const int64_t Ep = E_local > 0 ? E_local : E;
  TORCH_CHECK(pairs.size(0) >= (int64_t)T * k / MB + std::min<int64_t>(Ep, (int64_t)T * k), "moe_route_fused: pairs");
  if (T == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  const size_t smem = (size_t)4 * H * 2;
  // static shared memory of the top-k / pair-list phases + the token stage exceed the 48 KiB default
  moet_allow_max_smem(moe_route_fused_kernel);
  launch_k(moe_route_fused_kernel, (E + kRouteExperts - 1) / kRouteExperts, kRouteWarps * 32, smem, stream,
           (const __nv_bfloat16*)x.data_ptr(), T, H, (const __nv_bfloat16*)w.data_ptr(), E, logits.data_ptr<float>(),
           bias.has_value() && bias->defined() ? (const float*)bias->data_ptr<float>() : (const float*)nullptr,
           (int)k, sigmoid ? 1 : 0, (int)n_group, (int)topk_group, norm ? 1 : 0, (float)scaling,
           ids.data_ptr<int>(), wts.data_ptr<float>(), (int)MB, rank_scratch.data_ptr<int>(),
           sorted_tok.data_ptr<int>(), pos_of.data_ptr<int>(), (int4*)pairs.data_ptr<int>(), n_pairs.data_ptr<int>(),
           counter.data_ptr<int>(), status.data_ptr<int>(), (int)e_lo, (int)E_local, ep);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void router_logits(torch::Tensor x, torch::Tensor w, torch::Tensor out, c10::optional<torch::Tensor> part,
                   c10::optional<torch::Tensor> cnt) {
  const int T = x.size(0), H = x.size(1), E = w.size(0);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && x.is_contiguous() &&
              w.is_contiguous() && H % 256 == 0, "router_logits: bf16 contiguous, H % 256 == 0");
  if (T == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  // T > 64: tensor-core tiles of 64 tokens x 64 experts; when the tiles alone would leave the
  // GPU mostly idle (decode batches of tens of rows) K is sliced across grid.z, given scratch
  // for the partials (part >= ks * T * E floats) and the per-tile arrival counters (zeroed)
  if (T > 64 && E % 64 == 0 && H % 64 == 0 && out.is_contiguous()) {
    const int tiles = ((T + 63) / 64) * (E / 64);
    int ks = 1;
    const bool have = part.has_value() && part->defined() && cnt.has_value() && cnt->defined();
    if (have) {
      ks = std::max(1, std::min(H / 512, 64 / tiles));   // ~64 CTAs: short K loops, an 8-slice sum
      while (ks > 1 && ((int64_t)ks * T * E > part->numel() || (H / 64) % ks)) ks--;
      TORCH_CHECK(cnt->numel() >= tiles, "router_logits: counters");
    }
    launch_k(router_logits_mma_kernel, dim3((T + 63) / 64, E / 64, ks), 128, 0, stream,
             (const __nv_bfloat16*)x.data_ptr(), T, H, (const __nv_bfloat16*)w.data_ptr(), E, out.data_ptr<float>(),
             ks > 1 ? part->data_ptr<float>() : nullptr, ks > 1 ? cnt->data_ptr<int>() : nullptr, H / ks);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  launch_k(router_logits_kernel, (E + 7) / 8, 256, 0, stream, (const __nv_bfloat16*)x.data_ptr(), T, H,
                                                        (const __nv_bfloat16*)w.data_ptr(), E, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Padded variant: each expert's segment of the sorted rows starts at a multiple of MB
// (so a pair's rows are MB-aligned and contiguous); total rows -> n_rows[0].
// sorted_tok / pos_of must hold R / MB * MB + min(E, R) * MB rows.
void build_pairs_padded(torch::Tensor topk_ids, int64_t E, int64_t MB, torch::Tensor rank_scratch,
                        torch::Tensor sorted_tok, torch::Tensor pos_of, torch::Tensor pairs, torch::Tensor n_pairs,
                        torch::Tensor n_rows, torch::Tensor status, int64_t e_lo) {
  const int T = topk_ids.size(0), k = topk_ids.size(1), R = T * k;
  TORCH_CHECK(E <= kMaxE, "build_pairs_padded: E <= 512");
  const int64_t P = R / MB + std::min<int64_t>(E, R);
  TORCH_CHECK(pairs.size(0) >= P && sorted_tok.size(0) >= P * MB, "build_pairs_padded: buffers too small");
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_k(build_pairs_kernel, 1, 1024, 0, stream, topk_ids.data_ptr<int>(), R, k, (int)E, (int)MB,
                                             rank_scratch.data_ptr<int>(), sorted_tok.data_ptr<int>(),
                                             pos_of.data_ptr<int>(), (int4*)pairs.data_ptr<int>(),
                                             n_pairs.data_ptr<int>(), status.data_ptr<int>(), 1, n_rows.data_ptr<int>(),
                                             (int)std::max<int64_t>(e_lo, 0), e_lo >= 0 ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void build_pairs(torch::Tensor topk_ids, int64_t E, int64_t MB, torch::Tensor rank_scratch,
                 torch::Tensor sorted_tok, torch::Tensor pos_of, torch::Tensor pairs, torch::Tensor n_pairs,
                 torch::Tensor status, int64_t e_lo) {
  const int T = topk_ids.size(0), k = topk_ids.size(1), R = T * k;
  TORCH_CHECK(E <= kMaxE, "build_pairs: E <= 512");
  TORCH_CHECK(pairs.size(0) >= R / MB + std::min<int64_t>(E, R), "build_pairs: pairs buffer too small");
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_k(build_pairs_kernel, 1, 1024, 0, stream, topk_ids.data_ptr<int>(), R, k, (int)E, (int)MB,
                                             rank_scratch.data_ptr<int>(), sorted_tok.data_ptr<int>(),
                                             pos_of.data_ptr<int>(), (int4*)pairs.data_ptr<int>(),
                                             n_pairs.data_ptr<int>(), status.data_ptr<int>(), 0, (int*)nullptr,
                                             (int)std::max<int64_t>(e_lo, 0), e_lo >= 0 ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ep_recv_pairs(torch::Tensor desc, int64_t MB, torch::Tensor ids, torch::Tensor rank_scratch,
                   torch::Tensor sorted_tok, torch::Tensor pos_of, torch::Tensor pairs, torch::Tensor n_pairs,
                   torch::Tensor n_rows) {
  EpDesc d = ep_desc_from(desc);
  const int64_t R = (int64_t)d.world * d.cap;
  TORCH_CHECK(d.E_loc <= kMaxE, "ep_recv_pairs: at most 512 local experts");
  TORCH_CHECK(ids.numel() >= R && rank_scratch.numel() >= R && sorted_tok.numel() >= R && pos_of.numel() >= R &&
              pairs.size(0) >= R / MB + std::min<int64_t>(d.E_loc, R), "ep_recv_pairs: buffers too small");
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_k(ep_recv_pairs_kernel, 1, 1024, 0, stream, d, (int)MB, ids.data_ptr<int>(), rank_scratch.data_ptr<int>(),
           sorted_tok.data_ptr<int>(), pos_of.data_ptr<int>(), (int4*)pairs.data_ptr<int>(), n_pairs.data_ptr<int>(),
           n_rows.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------
// Scratch-free C entry point (declared in moe_route_noalloc.h): the same
// pair-list kernel, with its per-routing rank scratch in a static device array
// instead of a caller-provided buffer.
#include <mutex>
#include "moe_route_noalloc.h"

namespace moet_noalloc {
static __device__ __align__(256) int g_rank_scratch[MOET_NOALLOC_MAX_ROUTINGS];
constexpr int kMaxDevices = 128;
static int* g_scratch_addr[kMaxDevices];  // device address of g_rank_scratch, per device
static std::mutex g_mu;
}  // namespace moet_noalloc

extern "C" int moet_build_pairs_noalloc(const int* topk_ids, int num_tokens, int top_k, int num_experts,
                                        int rows_per_pair, int* sorted_tok, int* pos_of, int* pairs,
                                        int max_pairs, int* n_pairs, int* status, cudaStream_t stream) {
  using namespace moet_noalloc;
  if (!topk_ids || !sorted_tok || !pos_of || !pairs || !n_pairs || !status) return MOET_NOALLOC_EINVAL;
  if (num_tokens < 0 || top_k < 1 || top_k > 32 || num_experts < 1 || num_experts > moet::kMaxE ||
      rows_per_pair < 1)
    return MOET_NOALLOC_EINVAL;
  const long long R = (long long)num_tokens * top_k;
  if (R > MOET_NOALLOC_MAX_ROUTINGS) return MOET_NOALLOC_ETOOBIG;
  if ((long long)max_pairs < R / rows_per_pair + std::min<long long>(num_experts, R)) return MOET_NOALLOC_EINVAL;
  // the kernel writes each pair record as one 16-byte store
  if ((reinterpret_cast<uintptr_t>(pairs) & 15) != 0) return MOET_NOALLOC_EINVAL;
  int dev = 0;
  cudaError_t rc = cudaGetDevice(&dev);
  if (rc != cudaSuccess) return (int)rc;
  if (dev < 0 || dev >= kMaxDevices) return MOET_NOALLOC_EINVAL;
  int* scratch;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_addr[dev]) {
      void* p = nullptr;
      rc = cudaGetSymbolAddress(&p, g_rank_scratch);
      if (rc != cudaSuccess) return (int)rc;
      g_scratch_addr[dev] = static_cast<int*>(p);
    }
    scratch = g_scratch_addr[dev];
  }
  moet::build_pairs_kernel<<<1, 1024, 0, stream>>>(topk_ids, (int)R, top_k, num_experts, rows_per_pair, scratch,
                                                  sorted_tok, pos_of, reinterpret_cast<int4*>(pairs), n_pairs,
                                                  status);
  rc = cudaGetLastError();
  return rc == cudaSuccess ? MOET_NOALLOC_OK : (int)rc;
}
