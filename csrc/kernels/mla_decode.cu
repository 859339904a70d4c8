// MLA decode attention in the absorbed (latent) form, over a paged KV cache.
//
// Every query row (token t, head h) holds [q_lat (512) | q_rope (64)] where
// q_lat = W_uk^T q_nope; keys and values are the shared latent rows
// [c_kv (512) | k_rope (64)] of the cache, so all heads of a token share one
// KV stream (MQA-like).  One CTA handles all heads of one token for a
// contiguous share of its context ("split"); a combine kernel merges splits
// (flash-decoding) and emits the FP8 operand of the W_uv projection.
//
// KV cache (bf16): [blocks, 64, 584] bf16 -- 512 latent, 64 rope, 8 pad; the
// 1168-byte row stride makes ldmatrix conflict-free without a swizzle.  A
// whole 64-token block (74,752 B) is fetched by one cp.async.bulk
// (TMA bulk copy, no multicast) completing on an mbarrier; two buffers
// double-buffer the stream.  S = Q K^T and O += P V use mma.sync bf16
// m16n8k16 with fp32 accumulation; softmax is online (exp2 domain).
// All waits are bounded: on timeout the kernel records kTimeout in *status
// and returns instead of hanging.
#include "common.cuh"
#include "torch_glue.h"

namespace moet {

constexpr int kBS = 64;           // tokens per KV block
constexpr int kRow = 584;         // bf16 elements per cache row
constexpr int kLat = 512, kQK = 576;
constexpr int kBlockBytes = kBS * kRow * 2;
constexpr int kPRow = 72;         // P smem row (bf16), 144 B stride
constexpr int kRow4 = 352;        // NVFP4 cache row bytes: 256 e2m1 | 32 e4m3 scales | 64 e4m3 rope
constexpr int kBlockBytes4 = kBS * kRow4;

// e2m1 code -> value (sign in bit 3)
__device__ __constant__ float kE2M1[16] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f,
                                           -0.f, -0.5f, -1.f, -1.5f, -2.f, -3.f, -4.f, -6.f};

MOET_DEVICE uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
MOET_DEVICE void mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
MOET_DEVICE void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes));
}
MOET_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
MOET_DEVICE void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
MOET_DEVICE void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Bounded wait; returns false on timeout.
MOET_DEVICE bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  for (uint32_t it = 0; it < (1u << 22); it++)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

struct MlaDecodeArgs {
  const __nv_bfloat16* q; long long q_tok_stride;     // [T, Hh, 576]
  const __nv_bfloat16* kv; int n_blocks;               // [blocks, 64, 584]
  const int* block_table; int bt_stride;               // [seqs, max_blocks]
  const int* seq_of_tok; const int* pos_of_tok;        // [T]
  float* o_part; float* ml_part;                       // [S, T, Hh, 512], [S, T, Hh, 2]
  int T, Hh, nsplit;
  float scale_log2;                                    // softmax scale * log2(e)
  int* status;
  int nvfp4;                                           // cache rows are 352-byte NVFP4 (kv: uint8 [blocks, 64, 352])
  const int* sel; int sel_stride;                      // sparse mode: [T, topk] selected positions (-1 = none)
};

// Expand one staged NVFP4 block (64 rows x 352 B) into the bf16 tile [64][584]:
// latent = e2m1 * e4m3(block-16 scale) * 2^-6, rope = e4m3.
MOET_DEVICE void expand_nvfp4_block(const uint8_t* __restrict__ st, __nv_bfloat16* __restrict__ kvt) {
  for (int task = threadIdx.x; task < kBS * 16; task += blockDim.x) {
    const int r = task >> 4, c = task & 15;              // 16-byte chunk c = 32 latent dims
    const uint8_t* row = st + r * kRow4;
    const uint4 b = *reinterpret_cast<const uint4*>(row + c * 16);
    const float s0 = e4m3_to_f32(row[256 + 2 * c]) * 0.015625f, s1 = e4m3_to_f32(row[256 + 2 * c + 1]) * 0.015625f;
    const uint32_t w[4] = {b.x, b.y, b.z, b.w};
    uint32_t o[16];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const uint32_t byte = (w[i] >> (8 * j)) & 0xFF;
        const float sc = i < 2 ? s0 : s1;
        const __nv_bfloat162 v = __floats2bfloat162_rn(kE2M1[byte & 0xF] * sc, kE2M1[byte >> 4] * sc);
        o[i * 4 + j] = *reinterpret_cast<const uint32_t*>(&v);
      }
    uint4* dst = reinterpret_cast<uint4*>(kvt + (size_t)r * kRow + c * 32);
#pragma unroll
    for (int q = 0; q < 4; q++) dst[q] = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
  }
  for (int task = threadIdx.x; task < kBS * 8; task += blockDim.x) {
    const int r = task >> 3, c = task & 7;               // 8 rope dims per task
    const uint2 b = *reinterpret_cast<const uint2*>(st + r * kRow4 + 288 + c * 8);
    const uint32_t w[2] = {b.x, b.y};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const __nv_bfloat162 v0 = __floats2bfloat162_rn(e4m3_to_f32(w[i] & 0xFF), e4m3_to_f32((w[i] >> 8) & 0xFF));
      const __nv_bfloat162 v1 = __floats2bfloat162_rn(e4m3_to_f32((w[i] >> 16) & 0xFF), e4m3_to_f32(w[i] >> 24));
      o[2 * i] = *reinterpret_cast<const uint32_t*>(&v0);
      o[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&v1);
    }
    *reinterpret_cast<uint4*>(kvt + (size_t)r * kRow + kLat + c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <int MT>
__global__ void __launch_bounds__(256, 1) mla_decode_kernel(MlaDecodeArgs p) {
  pdl_entry();
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // bf16 cache: two 64-row tiles double-buffered by TMA.  NVFP4 cache: one bf16 tile
  // plus two 22.5 KB staging buffers (TMA fills one while the other is expanded).
  __nv_bfloat16* kvs = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  uint8_t* stage4 = smem_raw + (size_t)kBS * kRow * 2;
  __nv_bfloat16* qs = p.nvfp4 ? reinterpret_cast<__nv_bfloat16*>(stage4 + 2 * kBlockBytes4)
                              : kvs + 2 * kBS * kRow;                               // [16MT][584]
  __nv_bfloat16* ps = qs + 16 * MT * kRow;                                          // [16MT][72]
  float* red = reinterpret_cast<float*>(ps + 16 * MT * kPRow);                      // [8][16MT]
  uint64_t* bars = reinterpret_cast<uint64_t*>(red + 8 * 16 * MT);                  // [2]

  const int tok = blockIdx.x, split = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int R = 16 * MT;
  const int seq = p.seq_of_tok[tok];
  // dense: the first pos+1 positions; sparse: the selected positions (a -1 terminated prefix of sel[tok])
  int L = p.pos_of_tok[tok] + 1;
  const int* selr = p.sel ? p.sel + (size_t)tok * p.sel_stride : nullptr;
  if (selr) {
    __shared__ int nsel;
    if (threadIdx.x == 0) {
      int n = 0;
      while (n < p.sel_stride && selr[n] >= 0) n++;
      nsel = n;
    }
    __syncthreads();
    L = nsel;
  }
  const int ntiles = (L + kBS - 1) / kBS;
  const int tps = max(2, (ntiles + p.nsplit - 1) / p.nsplit);   // >= 2 tiles: keeps the KV double buffer busy
  const int t_begin = split * tps, t_end = min(ntiles, t_begin + tps);

  if (threadIdx.x == 0) { mbar_init(&bars[0], 1); mbar_init(&bars[1], 1); fence_proxy_async(); }
  // Q rows -> smem (rows >= Hh zero)
  for (int i = threadIdx.x; i < R * (kQK / 8); i += blockDim.x) {
    const int r = i / (kQK / 8), c = (i % (kQK / 8)) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < p.Hh) v = *reinterpret_cast<const uint4*>(p.q + (size_t)tok * p.q_tok_stride + (size_t)r * kQK + c);
    *reinterpret_cast<uint4*>(qs + r * kRow + c) = v;
  }
  __syncthreads();

  auto issue = [&](int tile, int buf) {
    if (selr) {     // gather the tile's selected rows one bulk copy each, all on one barrier
      const int rb = p.nvfp4 ? kRow4 : kRow * 2;
      mbar_expect_tx(&bars[buf], (uint32_t)(kBS * rb));
      uint8_t* dst = p.nvfp4 ? stage4 + (size_t)buf * kBlockBytes4
                             : reinterpret_cast<uint8_t*>(kvs + (size_t)buf * kBS * kRow);
      const int first = selr[0];
      for (int r = 0; r < kBS; r++) {
        int pos = tile * kBS + r < L ? selr[tile * kBS + r] : first;   // masked rows re-read a valid row
        int blk = p.block_table[(size_t)seq * p.bt_stride + pos / kBS];
        if (blk < 0 || blk >= p.n_blocks || pos < 0) { set_status(p.status, kBadIndex); blk = 0; pos = 0; }
        const size_t src_row = (size_t)blk * kBS + (pos % kBS);
        bulk_g2s(dst + (size_t)r * rb, reinterpret_cast<const uint8_t*>(p.kv) + src_row * rb, rb, &bars[buf]);
      }
      return;
    }
    int blk = p.block_table[(size_t)seq * p.bt_stride + tile];
    if (blk < 0 || blk >= p.n_blocks) { set_status(p.status, kBadIndex); blk = 0; }
    if (p.nvfp4) {
      mbar_expect_tx(&bars[buf], kBlockBytes4);
      bulk_g2s(stage4 + (size_t)buf * kBlockBytes4,
               reinterpret_cast<const uint8_t*>(p.kv) + (size_t)blk * kBlockBytes4, kBlockBytes4, &bars[buf]);
    } else {
      mbar_expect_tx(&bars[buf], kBlockBytes);
      bulk_g2s(kvs + (size_t)buf * kBS * kRow, p.kv + (size_t)blk * kBS * kRow, kBlockBytes, &bars[buf]);
    }
  };
  if (threadIdx.x == 0 && t_begin < t_end) issue(t_begin, 0);

  float o[MT][8][4];
#pragma unroll
  for (int a = 0; a < MT; a++)
#pragma unroll
    for (int b = 0; b < 8; b++) o[a][b][0] = o[a][b][1] = o[a][b][2] = o[a][b][3] = 0.f;
  float m_run[MT][2], l_run[MT][2];
#pragma unroll
  for (int a = 0; a < MT; a++) { m_run[a][0] = m_run[a][1] = -INFINITY; l_run[a][0] = l_run[a][1] = 0.f; }

  uint32_t phase[2] = {0, 0};
  bool ok = true;
  for (int tile = t_begin; tile < t_end; tile++) {
    const int buf = (tile - t_begin) & 1;
    if (threadIdx.x == 0 && tile + 1 < t_end) { fence_proxy_async(); issue(tile + 1, buf ^ 1); }
    if (!mbar_wait_bounded(&bars[buf], phase[buf])) { ok = false; }
    phase[buf] ^= 1;
    if (!__syncthreads_and(ok)) { set_status(p.status, kTimeout); return; }
    const __nv_bfloat16* kvt = kvs + (size_t)buf * kBS * kRow;
    if (p.nvfp4) {
      expand_nvfp4_block(stage4 + (size_t)buf * kBlockBytes4, kvs);
      __syncthreads();
      kvt = kvs;
    }

    // ---- S = Q K^T for positions [8w, 8w+8) of the tile ----
    float s[MT][4];
#pragma unroll
    for (int a = 0; a < MT; a++) s[a][0] = s[a][1] = s[a][2] = s[a][3] = 0.f;
#pragma unroll 4
    for (int kk = 0; kk < kQK / 16; kk++) {
      uint32_t bfrag[2];
      ldmatrix_x2(bfrag, kvt + (size_t)(warp * 8 + (lane & 7)) * kRow + kk * 16 + ((lane >> 3) & 1) * 8);
#pragma unroll
      for (int a = 0; a < MT; a++) {
        uint32_t afrag[4];
        ldmatrix_x4(afrag, qs + (size_t)(a * 16 + (lane & 15)) * kRow + kk * 16 + (lane >> 4) * 8);
        mma_bf16_16816(s[a], afrag, bfrag[0], bfrag[1]);
      }
    }
    // scale + mask, per-warp row max
    const int pbase = tile * kBS + warp * 8 + 2 * t;
    float tmax[MT][2];
#pragma unroll
    for (int a = 0; a < MT; a++) {
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int pos = pbase + (i & 1);
        s[a][i] = pos < L ? s[a][i] * p.scale_log2 : -INFINITY;
      }
      tmax[a][0] = fmaxf(s[a][0], s[a][1]);
      tmax[a][1] = fmaxf(s[a][2], s[a][3]);
#pragma unroll
      for (int h = 0; h < 2; h++) {
        tmax[a][h] = fmaxf(tmax[a][h], __shfl_xor_sync(0xffffffffu, tmax[a][h], 1));
        tmax[a][h] = fmaxf(tmax[a][h], __shfl_xor_sync(0xffffffffu, tmax[a][h], 2));
      }
      if (t == 0) { red[warp * R + a * 16 + g] = tmax[a][0]; red[warp * R + a * 16 + g + 8] = tmax[a][1]; }
    }
    __syncthreads();
    float m_new[MT][2], alpha[MT][2];
#pragma unroll
    for (int a = 0; a < MT; a++)
#pragma unroll
      for (int h = 0; h < 2; h++) {
        float mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < 8; w++) mx = fmaxf(mx, red[w * R + a * 16 + g + 8 * h]);
        m_new[a][h] = fmaxf(m_run[a][h], mx);
        alpha[a][h] = m_new[a][h] == -INFINITY ? 1.f : exp2f(m_run[a][h] - m_new[a][h]);
      }
    __syncthreads();  // red reused for row sums
    // P = exp2(S - m), to smem as bf16; partial row sums
#pragma unroll
    for (int a = 0; a < MT; a++) {
      float e0 = m_new[a][0] == -INFINITY ? 0.f : exp2f(s[a][0] - m_new[a][0]);
      float e1 = m_new[a][0] == -INFINITY ? 0.f : exp2f(s[a][1] - m_new[a][0]);
      float e2 = m_new[a][1] == -INFINITY ? 0.f : exp2f(s[a][2] - m_new[a][1]);
      float e3 = m_new[a][1] == -INFINITY ? 0.f : exp2f(s[a][3] - m_new[a][1]);
      __nv_bfloat162 p01 = __floats2bfloat162_rn(e0, e1), p23 = __floats2bfloat162_rn(e2, e3);
      *reinterpret_cast<__nv_bfloat162*>(ps + (a * 16 + g) * kPRow + warp * 8 + 2 * t) = p01;
      *reinterpret_cast<__nv_bfloat162*>(ps + (a * 16 + g + 8) * kPRow + warp * 8 + 2 * t) = p23;
      // row sums of the rounded probabilities (what the PV product uses)
      float r0 = __low2float(p01) + __high2float(p01), r1 = __low2float(p23) + __high2float(p23);
      r0 += __shfl_xor_sync(0xffffffffu, r0, 1); r0 += __shfl_xor_sync(0xffffffffu, r0, 2);
      r1 += __shfl_xor_sync(0xffffffffu, r1, 1); r1 += __shfl_xor_sync(0xffffffffu, r1, 2);
      if (t == 0) { red[warp * R + a * 16 + g] = r0; red[warp * R + a * 16 + g + 8] = r1; }
    }
    __syncthreads();
#pragma unroll
    for (int a = 0; a < MT; a++)
#pragma unroll
      for (int h = 0; h < 2; h++) {
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++) sum += red[w * R + a * 16 + g + 8 * h];
        l_run[a][h] = l_run[a][h] * alpha[a][h] + sum;
        m_run[a][h] = m_new[a][h];
      }
#pragma unroll
    for (int a = 0; a < MT; a++)
#pragma unroll
      for (int nt = 0; nt < 8; nt++) {
        o[a][nt][0] *= alpha[a][0]; o[a][nt][1] *= alpha[a][0];
        o[a][nt][2] *= alpha[a][1]; o[a][nt][3] *= alpha[a][1];
      }
    // ---- O += P V for latent dims [64w, 64w+64) ----
#pragma unroll
    for (int kk = 0; kk < kBS / 16; kk++) {
      uint32_t afrag[MT][4];
#pragma unroll
      for (int a = 0; a < MT; a++)
        ldmatrix_x4(afrag[a], ps + (size_t)(a * 16 + (lane & 15)) * kPRow + kk * 16 + (lane >> 4) * 8);
#pragma unroll
      for (int np = 0; np < 4; np++) {  // pairs of n8 tiles
        const int d0 = warp * 64 + np * 16;
        const int prow = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int dcol = d0 + (lane >> 4) * 8;
        uint32_t b[4];
        ldmatrix_x4_trans(b, kvt + (size_t)prow * kRow + dcol);
#pragma unroll
        for (int a = 0; a < MT; a++) {
          mma_bf16_16816(o[a][2 * np], afrag[a], b[0], b[1]);
          mma_bf16_16816(o[a][2 * np + 1], afrag[a], b[2], b[3]);
        }
      }
    }
    __syncthreads();  // buffer + P free for the next tile
  }
  // ---- write partial state ----
  const size_t base = ((size_t)split * p.T + tok) * p.Hh;
#pragma unroll
  for (int a = 0; a < MT; a++)
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int row = a * 16 + g + 8 * h;
      if (row >= p.Hh) continue;
      float* op = p.o_part + (base + row) * kLat + warp * 64;
#pragma unroll
      for (int nt = 0; nt < 8; nt++)
        *reinterpret_cast<float2*>(op + nt * 8 + 2 * t) = make_float2(o[a][nt][2 * h], o[a][nt][2 * h + 1]);
      if (warp == 0 && t == 0) {
        p.ml_part[(base + row) * 2] = m_run[a][h];
        p.ml_part[(base + row) * 2 + 1] = l_run[a][h];
      }
    }
}

// Merge splits; emit bf16 [T, Hh, 512] and/or e4m3 + UE8M0 per-64 scales.
__global__ void mla_combine_kernel(const float* __restrict__ o_part, const float* __restrict__ ml_part,
                                   int S, int TH, __nv_bfloat16* __restrict__ out,
                                   uint8_t* __restrict__ q, uint8_t* __restrict__ qs) {
  pdl_entry();
  const int row = blockIdx.x;  // (t, h)
  float M = -INFINITY;
  for (int s = 0; s < S; s++) M = fmaxf(M, ml_part[((size_t)s * TH + row) * 2]);
  float denom = 0.f;
  for (int s = 0; s < S; s++) {
    const float m = ml_part[((size_t)s * TH + row) * 2];
    if (m != -INFINITY) denom += exp2f(m - M) * ml_part[((size_t)s * TH + row) * 2 + 1];
  }
  const float inv = denom > 0.f ? 1.f / denom : 0.f;
  // 64 threads x 8 dims
  const int d0 = threadIdx.x * 8;
  float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int s = 0; s < S; s++) {
    const float m = ml_part[((size_t)s * TH + row) * 2];
    if (m == -INFINITY) continue;
    const float w = exp2f(m - M) * inv;
    const float* op = o_part + ((size_t)s * TH + row) * kLat + d0;
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = fmaf(w, op[i], v[i]);
  }
#pragma unroll
  for (int i = 0; i < 8; i++) v[i] = __bfloat162float(__float2bfloat16(v[i]));
  if (out) {
#pragma unroll
    for (int i = 0; i < 8; i++) out[(size_t)row * kLat + d0 + i] = __float2bfloat16(v[i]);
  }
  if (q) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const uint32_t e = ue8m0_for_amax(amax);
    const float invs = (e >= 1 && e <= 253) ? __uint_as_float((254u - e) << 23) : 0.f;
    uint8_t b[8];
#pragma unroll
    for (int i = 0; i < 8; i++) b[i] = f32_to_e4m3(v[i] * invs);
    *reinterpret_cast<uint2*>(q + (size_t)row * kLat + d0) = *reinterpret_cast<uint2*>(b);
    if ((threadIdx.x & 7) == 0) qs[(size_t)row * (kLat / 64) + d0 / 64] = (uint8_t)e;
  }
}

// Split merge fused with the absorbed value projection and its quantisation:
// one CTA per head h merges the S partial states of every token into o_lat
// (bf16-rounded, kept in shared memory), applies W_uv[h] (128 x 512, e4m3 with
// UE8M0 128x128 block scales) and writes ov[t, h*128 + j] as e4m3 with UE8M0
// per-64 scales -- the input of the o projection.
constexpr int kTC = 16;   // tokens per smem chunk
__global__ void __launch_bounds__(256) mla_combine_uv_kernel(const float* __restrict__ o_part,
                                                             const float* __restrict__ ml_part, int S, int T, int Hh,
                                                             const uint8_t* __restrict__ wuv,
                                                             const uint8_t* __restrict__ swuv,
                                                             uint8_t* __restrict__ q, uint8_t* __restrict__ qs,
                                                             int VD) {
  __shared__ __align__(16) float olat[kTC][kLat];
  __shared__ float ov[kTC][64];
  __shared__ float wgt[kTC][32];
  __shared__ int nact[kTC];
  const int h = blockIdx.x, TH = T * Hh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint8_t* W = wuv + (size_t)h * VD * kLat;
  const uint8_t* SW = swuv + (size_t)h * (VD / 128) * (kLat / 128);   // [VD/128, 4] block scales of this head
  // CTA (head h, group hv) computes output rows [64 hv, 64 hv + 64) -- exactly one quantisation group;
  // thread (row j, quarter qk) owns W[j][128*qk .. +128) -- one scale block; immutable, so it is
  // loaded before the dependency wait
  const int hv = blockIdx.y;
  const int jl = threadIdx.x >> 2, j = hv * 64 + jl, qk = threadIdx.x & 3, nwarps = blockDim.x >> 5;
  uint4 wrow[8];
#pragma unroll
  for (int u = 0; u < 8; u++)
    wrow[u] = __ldg(reinterpret_cast<const uint4*>(W + (size_t)j * kLat + qk * 128) + u);
  const float wsc = ue8m0_to_float(__ldg(SW + (j >> 7) * (kLat / 128) + qk));
  pdl_entry();
  const int tbeg = blockIdx.z * kTC, tend = min(T, tbeg + kTC);
  for (int t0 = tbeg; t0 < tend; t0 += kTC) {
    const int nt = min(kTC, T - t0);
    // split weights exp2(m_s - M) / sum: one warp per token (S <= 32)
    for (int tt = warp; tt < nt; tt += nwarps) {
      const int row = (t0 + tt) * Hh + h;
      const float m = lane < S ? ml_part[((size_t)lane * TH + row) * 2] : -INFINITY;
      const float l = lane < S ? ml_part[((size_t)lane * TH + row) * 2 + 1] : 0.f;
      const float M = warp_max(m);
      const float e = m == -INFINITY ? 0.f : exp2f(m - M);
      const float den = warp_sum(e * l);
      wgt[tt][lane] = den > 0.f ? e / den : 0.f;
      // active splits form a prefix (each split takes the next range of KV tiles)
      const unsigned act = __ballot_sync(0xffffffffu, m != -INFINITY);
      if (lane == 0) nact[tt] = 32 - __clz(act);
    }
    __syncthreads();
    // merge: each thread owns 4 consecutive dims of one token; loads of 4 splits in flight
    for (int i = threadIdx.x; i < nt * (kLat / 4); i += blockDim.x) {
      const int tt = i / (kLat / 4), d = (i % (kLat / 4)) * 4;
      const int row = (t0 + tt) * Hh + h;
      const int na = nact[tt];
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int sp0 = 0; sp0 < na; sp0 += 4) {
        float4 pv[4];
#pragma unroll
        for (int u = 0; u < 4; u++)
          pv[u] = sp0 + u < na ? *reinterpret_cast<const float4*>(o_part + ((size_t)(sp0 + u) * TH + row) * kLat + d)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const float w = sp0 + u < na ? wgt[tt][sp0 + u] : 0.f;
          v.x = fmaf(w, pv[u].x, v.x); v.y = fmaf(w, pv[u].y, v.y);
          v.z = fmaf(w, pv[u].z, v.z); v.w = fmaf(w, pv[u].w, v.w);
        }
      }
      float* dst = &olat[tt][d];
      dst[0] = __bfloat162float(__float2bfloat16(v.x)); dst[1] = __bfloat162float(__float2bfloat16(v.y));
      dst[2] = __bfloat162float(__float2bfloat16(v.z)); dst[3] = __bfloat162float(__float2bfloat16(v.w));
    }
    __syncthreads();
    // ov[t][j] = sum_k W[j][k] * olat[t][k]: four threads per row, joined by two shuffles
    for (int tt = 0; tt < nt; tt++) {
      const float4* op = reinterpret_cast<const float4*>(&olat[tt][qk * 128]);
      float acc = 0.f;
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const uint8_t* wb = reinterpret_cast<const uint8_t*>(&wrow[u]);
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float4 o4 = op[u * 4 + i];
          acc = fmaf(e4m3_to_f32(wb[4 * i]), o4.x, fmaf(e4m3_to_f32(wb[4 * i + 1]), o4.y,
                fmaf(e4m3_to_f32(wb[4 * i + 2]), o4.z, fmaf(e4m3_to_f32(wb[4 * i + 3]), o4.w, acc))));
        }
      }
      float v = acc * wsc;
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      if (qk == 0) ov[tt][jl] = __bfloat162float(__float2bfloat16(v));
    }
    __syncthreads();
    // quantise: one warp per token (this CTA's 64 outputs form one group), 2 values per lane
    for (int tt = warp; tt < nt; tt += nwarps) {
      const int g0 = hv * 64;
      const float a = ov[tt][2 * lane], b = ov[tt][2 * lane + 1];
      const float amax = warp_max(fmaxf(fabsf(a), fabsf(b)));
      const uint32_t e = ue8m0_for_amax(amax);
      const float inv = (e >= 1 && e <= 253) ? __uint_as_float((254u - e) << 23) : 0.f;
      const size_t col = (size_t)h * VD + g0;
      uint8_t* dq = q + (size_t)(t0 + tt) * Hh * VD + col + 2 * lane;
      dq[0] = f32_to_e4m3(a * inv);
      dq[1] = f32_to_e4m3(b * inv);
      if (lane == 0) qs[(size_t)(t0 + tt) * (Hh * VD / 64) + col / 64] = (uint8_t)e;
    }
    __syncthreads();
  }
}

}  // namespace moet

using namespace moet;

void mla_combine_uv(torch::Tensor o_part, torch::Tensor ml_part, torch::Tensor wuv, torch::Tensor swuv,
                    torch::Tensor q, torch::Tensor qs) {
  const int S = o_part.size(0), T = o_part.size(1), Hh = o_part.size(2);
  TORCH_CHECK(o_part.size(3) == kLat && S <= 32 && o_part.is_contiguous() && ml_part.is_contiguous(),
              "mla_combine_uv: o_part [S<=32, T, Hh, 512] contiguous");
  const int VD = wuv.size(1);
  TORCH_CHECK(wuv.dim() == 3 && wuv.size(0) == Hh && VD % 128 == 0 && VD <= 512 && wuv.size(2) == kLat &&
              wuv.is_contiguous(), "mla_combine_uv: W_uv [Hh, VD (128 | 256 ...), 512]");
  TORCH_CHECK(swuv.numel() == (int64_t)Hh * (VD / 128) * (kLat / 128) && swuv.is_contiguous(),
              "mla_combine_uv: W_uv scales [Hh, VD/128, 4]");
  TORCH_CHECK(q.is_contiguous() && q.size(-1) * (q.dim() == 3 ? q.size(1) : 1) == (int64_t)Hh * VD, "mla_combine_uv: out");
  if (T == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_k(mla_combine_uv_kernel, dim3(Hh, VD / 64, (T + kTC - 1) / kTC), 256, 0, stream, o_part.data_ptr<float>(), ml_part.data_ptr<float>(), S, T, Hh,
           (const uint8_t*)wuv.data_ptr(), (const uint8_t*)swuv.data_ptr(), (uint8_t*)q.data_ptr(),
           (uint8_t*)qs.data_ptr(), VD);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mla_decode(torch::Tensor q, torch::Tensor kv, torch::Tensor block_table, torch::Tensor seq_of_tok,
                torch::Tensor pos_of_tok, torch::Tensor o_part, torch::Tensor ml_part, double scale,
                torch::Tensor status, c10::optional<torch::Tensor> sel) {
  const int T = q.size(0), Hh = q.size(1);
  TORCH_CHECK(q.size(2) == kQK && q.stride(2) == 1 && q.stride(1) == kQK, "mla_decode: q [T, Hh, 576]");
  const bool nv4 = kv.scalar_type() == at::kByte;
  TORCH_CHECK(kv.size(1) == kBS && kv.size(2) == (nv4 ? kRow4 : kRow) && kv.is_contiguous(),
              "mla_decode: kv [blocks,64,584] bf16 or [blocks,64,352] uint8 (NVFP4)");
  TORCH_CHECK(Hh <= 32, "mla_decode: at most 32 heads per rank");
  const int S = o_part.size(0);
  TORCH_CHECK(o_part.size(1) == T && o_part.size(2) == Hh && o_part.size(3) == kLat, "mla_decode: o_part shape");
  if (T == 0) return;
  MlaDecodeArgs p;
  p.q = (const __nv_bfloat16*)q.data_ptr(); p.q_tok_stride = q.stride(0);
  p.kv = (const __nv_bfloat16*)kv.data_ptr(); p.n_blocks = kv.size(0);
  p.block_table = block_table.data_ptr<int>(); p.bt_stride = block_table.stride(0);
  p.seq_of_tok = seq_of_tok.data_ptr<int>(); p.pos_of_tok = pos_of_tok.data_ptr<int>();
  p.o_part = o_part.data_ptr<float>(); p.ml_part = ml_part.data_ptr<float>();
  p.T = T; p.Hh = Hh; p.nsplit = S;
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  p.nvfp4 = nv4 ? 1 : 0;
  p.sel = nullptr; p.sel_stride = 0;
  if (sel.has_value() && sel->defined()) {
    TORCH_CHECK(sel->scalar_type() == at::kInt && sel->dim() == 2 && sel->size(0) == T && sel->stride(1) == 1,
                "mla_decode: sel [T, topk] int32");
    p.sel = sel->data_ptr<int>(); p.sel_stride = sel->stride(0);
    TORCH_CHECK(sel->size(1) == p.sel_stride, "mla_decode: sel rows must be contiguous");
  }
  p.status = status.data_ptr<int>();
  auto stream = at::cuda::getCurrentCUDAStream();
  dim3 grid(T, S);
  if (Hh <= 16) {
    const int MT = 1;
    size_t smem = (size_t)((nv4 ? 1 : 2) * kBS * kRow + 16 * MT * kRow + 16 * MT * kPRow) * 2 + 8 * 16 * MT * 4 + 16 +
                  (nv4 ? 2 * kBlockBytes4 : 0);
    moet_allow_max_smem(mla_decode_kernel<1>);
    launch_k(mla_decode_kernel<1>, grid, 256, smem, stream, p);
  } else {
    const int MT = 2;
    size_t smem = (size_t)((nv4 ? 1 : 2) * kBS * kRow + 16 * MT * kRow + 16 * MT * kPRow) * 2 + 8 * 16 * MT * 4 + 16 +
                  (nv4 ? 2 * kBlockBytes4 : 0);
    moet_allow_max_smem(mla_decode_kernel<2>);
    launch_k(mla_decode_kernel<2>, grid, 256, smem, stream, p);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mla_combine(torch::Tensor o_part, torch::Tensor ml_part, c10::optional<torch::Tensor> out,
                 c10::optional<torch::Tensor> q, c10::optional<torch::Tensor> qs) {
  const int S = o_part.size(0), TH = o_part.size(1) * o_part.size(2);
  if (TH == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_k(mla_combine_kernel, TH, 64, 0, stream, o_part.data_ptr<float>(), ml_part.data_ptr<float>(), S, TH,
                                            (__nv_bfloat16*)opt_ptr(out), (uint8_t*)opt_ptr(q),
                                            (uint8_t*)opt_ptr(qs));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
