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
//   (w >> s) & 0x3333 is directly a prmt selector; one prmt over the fixed
//   4-entry e4m3 lookup word yields four e4m3 weights.
// * Scales: each k32 MMA accumulates into its own fragment, and the UE8M0
//   block scale (an exact power of two) and the activation scale are applied
//   with FMAs, exactly as the format defines the dequantised weight.
// * Misses (slot < 0) write zero rows and bump a miss counter.
// * Delta tier, two containers.  Direct-8: the slot holds e4m3 bytes already in
//   A-fragment register order (no decode).  Split FP4 ("quintal", w4q): the slot
//   holds only a radix-5 refinement plane read against the resident 2-bit base
//   (codes and scales of the base slot); per group of 4 codes a 10-bit word gives
//   the e2m1 magnitude index inside each code's class ({0,.5,1,1.5,2} or
//   {3,4,6}), so the decode rebuilds the exact MXFP4 value: digits from a
//   per-warp 625-entry table, class offset from the code bits, one prmt over the
//   e2m1 -> e4m3 magnitude pool, the sign bit from the base level.
#include "common.cuh"
#include "ep_a2a.cuh"
#include "symm.cuh"
#include "torch_glue.h"

namespace moet {

struct W2Args {
  const uint8_t* A; const uint8_t* sA; long long a_stride;  // activations (w2 layout), row stride bytes
  const int* gather;            // sorted row -> activation row (nullptr: identity)
  const int4* pairs; const int* n_pairs;
  const uint8_t* pool; long long slot_bytes; long long codes_off, scale_off;
  const int* slot_table;        // expert -> slot (< 0: miss)
  float* out; long long out_stride;
  int N, K;
  int* miss_count;
  // FP4 delta tier (direct-8 planes: e4m3 bytes in A-fragment order + UE8M0 block-32
  // scales); an expert with a delta slot >= 0 is served from it instead of the 2-bit slot
  const uint8_t* pool8; long long slot_bytes8, codes_off8, scale_off8;
  const int* slot_table8;
  int quintal;                  // delta slots hold split-FP4 refinement planes (base codes + scales stay in use)
  // expert parallelism, return leg: output row r (sorted) goes to the source rank's return
  // row ret_rows[r] = src * cap + i (peer store), and the grid publishes a return flag
  int ep_on; const int* ret_rows; EpDesc ep;
  // K slices (grid.z): slice z covers 64-k chunks [z * cps, (z + 1) * cps) and writes out + z * part_stride
  int cps; long long part_stride;
};

// 10-bit quintal word -> (d0 | d2 << 4) | (d1 | d3 << 4) << 8; x / 5 = (x * 0x334) >> 12 for x < 1024
MOET_DEVICE uint32_t quintal_digit_word(uint32_t w) {
  const uint32_t q1 = (w * 0x334u) >> 12, d0 = w - 5u * q1;
  const uint32_t q2 = (q1 * 0x334u) >> 12, d1 = q1 - 5u * q2;
  const uint32_t q3 = (q2 * 0x334u) >> 12, d2 = q2 - 5u * q3;
  return (d0 | (d2 << 4)) | ((d1 | (q3 << 4)) << 8);
}

// One A-fragment register of split FP4: csel = the 4 code nibbles of the register (as the
// 2-bit decode selects them), Ta / Tb = the digit words of its two groups, mode picks the
// even (0x0040) or odd (0x0051) code positions.
MOET_DEVICE uint32_t quintal_reg(uint32_t csel, uint32_t Ta, uint32_t Tb, uint32_t mode) {
  constexpr uint32_t L = 0x4838B8C8u, MLO = 0x3C383000u, MHI = 0x4C484440u;
  const uint32_t base = prmt(L, L, csel);
  const uint32_t dsel = prmt(Ta, Tb, mode);
  const uint32_t big = ~(csel ^ (csel >> 1)) & 0x1111u;      // codes 0 and 3: the {3, 4, 6} class
  return prmt(MLO, MHI, dsel + 5u * big) | (base & 0x80808080u);
}

// Destination of output row r0 + j: the local out matrix, or under expert parallelism the
// source rank's return row in peer memory.
MOET_DEVICE float* w2_out_row(const W2Args& p, int r) {
  if (!p.ep_on) return p.out + (size_t)blockIdx.z * p.part_stride + (size_t)r * p.out_stride;
  const int rr = p.ret_rows[r], src = rr / p.ep.cap;
  return ep_ret(p.ep, src) + (size_t)(rr - src * p.ep.cap) * p.ep.H;
}

template <int NT>
__device__ __forceinline__ void moe_w2_gemv_body(const W2Args& p) {
  pdl_entry();
  const int pi = blockIdx.y;
  if (pi >= *p.n_pairs) return;
  const int4 pr = p.pairs[pi];
  const int e = pr.x, r0 = pr.y, nrows = pr.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int nb = blockIdx.x * (blockDim.x >> 5) + warp;  // 16-row block
  if (nb * 16 >= p.N) return;
  const int slot8 = p.slot_table8 ? p.slot_table8[e] : -1;
  const bool split = p.quintal && slot8 >= 0;                 // refinement over the base: the base must be resident
  const int slot = slot8 >= 0 && !p.quintal ? slot8 : p.slot_table[e];
  if (slot < 0) {
    if (blockIdx.x == 0 && blockIdx.z == 0 && threadIdx.x == 0 && p.miss_count) atomicAdd(p.miss_count, 1);
    for (int j = 0; j < nrows; j++)
      if (lane < 16) w2_out_row(p, r0 + j)[nb * 16 + lane] = 0.f;
    return;
  }
  const int KC = p.K >> 6, KS = p.K >> 5;
  const int c_begin = blockIdx.z * p.cps, c_end = min(KC, c_begin + p.cps);   // this CTA's K slice
  const bool direct = slot8 >= 0 && !p.quintal;
  const uint8_t* base = direct ? p.pool8 + (size_t)slot8 * p.slot_bytes8 : p.pool + (size_t)slot * p.slot_bytes;
  const uint8_t* codes = direct ? base + p.codes_off8 + (size_t)nb * KC * 1024 + lane * 32
                                : base + p.codes_off + (size_t)nb * KC * 256 + lane * 8;
  const uint8_t* sc = base + (direct ? p.scale_off8 : p.scale_off) + (size_t)nb * KS * 16;
  const uint8_t* qrec = split ? p.pool8 + (size_t)slot8 * p.slot_bytes8 + p.codes_off8 + (size_t)nb * KC * 320 : nullptr;

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

  // The warp's scale plane (16 rows x K/32 bytes, contiguous) -> shared memory.
  extern __shared__ __align__(16) uint8_t scale_smem[];
  uint8_t* ss = scale_smem + warp * 16 * KS;
  for (int i = lane; i < KS; i += 32)
    reinterpret_cast<uint4*>(ss)[i] = __ldg(reinterpret_cast<const uint4*>(sc) + i);
  // split FP4: this warp's digit table (after every warp's scale stage: (blockDim/32) * 16 * KS bytes)
  uint16_t* qlut = reinterpret_cast<uint16_t*>(scale_smem + (blockDim.x >> 5) * 16 * KS) + warp * 640;
  if (split)
    for (int w = lane; w < 625; w += 32) qlut[w] = (uint16_t)quintal_digit_word(w);
  __syncwarp();

  // Chunks are streamed in batches of U: all code loads of a batch are issued
  // before any of them is consumed.  Decode uses one fixed lookup word (code ->
  // e4m3 level), one prmt per 4 codes; each k32 MMA gets its own accumulator
  // fragment and the two block scales are applied with FMAs.
  constexpr uint32_t L = 0x4838B8C8u;   // e4m3 {-4, -1, +1, +4}
  constexpr int U = 8;
  auto mma_chunk = [&](int c, const uint32_t (&A0)[4], const uint32_t (&A1)[4]) {
    const uint8_t* s = ss + c * 32;
    const float sga = ue8m0_to_float(s[g]), sha = ue8m0_to_float(s[g + 8]);
    const float sgb = ue8m0_to_float(s[16 + g]), shb = ue8m0_to_float(s[24 + g]);
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
      uint2 xa = make_uint2(0, 0), xb = make_uint2(0, 0);
      if (xr[nt] >= 0) {
        const uint8_t* xp = xbase + (size_t)xr[nt] * p.a_stride + (size_t)c * 64;
        xa = __ldg(reinterpret_cast<const uint2*>(xp));
        xb = __ldg(reinterpret_cast<const uint2*>(xp + 32));
      }
      float da[4] = {0.f, 0.f, 0.f, 0.f}, db[4] = {0.f, 0.f, 0.f, 0.f};
      mma_e4m3_16832(da, A0, xa.x, xa.y, da);
      mma_e4m3_16832(db, A1, xb.x, xb.y, db);
      const float as0 = sr0[nt] >= 0 ? ue8m0_to_float(__ldg(p.sA + (size_t)sr0[nt] * KC64 + c)) : 0.f;
      const float as1 = sr1[nt] >= 0 ? ue8m0_to_float(__ldg(p.sA + (size_t)sr1[nt] * KC64 + c)) : 0.f;
      acc[nt][0] = fmaf(fmaf(da[0], sga, db[0] * sgb), as0, acc[nt][0]);
      acc[nt][1] = fmaf(fmaf(da[1], sga, db[1] * sgb), as1, acc[nt][1]);
      acc[nt][2] = fmaf(fmaf(da[2], sha, db[2] * shb), as0, acc[nt][2]);
      acc[nt][3] = fmaf(fmaf(da[3], sha, db[3] * shb), as1, acc[nt][3]);
    }
  };
  if (direct) {     // delta tier: the A-fragments are stored as e4m3 bytes, no decode
    constexpr int UD = 2;
    for (int c0 = c_begin; c0 < c_end; c0 += UD) {
      uint4 w0[UD], w1[UD];
#pragma unroll
      for (int u = 0; u < UD; u++)
        if (c0 + u < c_end) {
          w0[u] = ldg_stream_u4(codes + (size_t)(c0 + u) * 1024);
          w1[u] = ldg_stream_u4(codes + (size_t)(c0 + u) * 1024 + 16);
        }
#pragma unroll
      for (int u = 0; u < UD; u++) {
        if (c0 + u >= c_end) break;
        const uint32_t A0[4] = {w0[u].x, w0[u].y, w0[u].z, w0[u].w};
        const uint32_t A1[4] = {w1[u].x, w1[u].y, w1[u].z, w1[u].w};
        mma_chunk(c0 + u, A0, A1);
      }
    }
  } else if (split) {
    constexpr int UQ = 2;
    for (int c0 = c_begin; c0 < c_end; c0 += UQ) {
      uint2 wv[UQ], qv[UQ];
      uint32_t qh[UQ];
#pragma unroll
      for (int u = 0; u < UQ; u++)
        if (c0 + u < c_end) {
          wv[u] = ldg_stream_u2(codes + (size_t)(c0 + u) * 256);
          qv[u] = ldg_stream_u2(qrec + (size_t)(c0 + u) * 320 + lane * 8);
          qh[u] = __ldg(reinterpret_cast<const unsigned short*>(qrec + (size_t)(c0 + u) * 320 + 256 + lane * 2));
        }
#pragma unroll
      for (int u = 0; u < UQ; u++) {
        if (c0 + u >= c_end) break;
        const uint32_t lo = wv[u].x, hi = wv[u].y, r0 = qv[u].x, r1 = qv[u].y, h = qh[u];
        // the lane's 8 ten-bit words (80-bit little-endian record), one per group of 4 codes
        uint32_t T[8];
        T[0] = qlut[r0 & 0x3FFu];
        T[1] = qlut[(r0 >> 10) & 0x3FFu];
        T[2] = qlut[(r0 >> 20) & 0x3FFu];
        T[3] = qlut[__funnelshift_r(r0, r1, 30) & 0x3FFu];
        T[4] = qlut[(r1 >> 8) & 0x3FFu];
        T[5] = qlut[(r1 >> 18) & 0x3FFu];
        T[6] = qlut[__funnelshift_r(r1, h, 28) & 0x3FFu];
        T[7] = qlut[(h >> 6) & 0x3FFu];
        const uint32_t A0[4] = {quintal_reg(lo & 0x3333u, T[0], T[1], 0x0040u),
                                quintal_reg(hi & 0x3333u, T[4], T[5], 0x0040u),
                                quintal_reg((lo >> 2) & 0x3333u, T[0], T[1], 0x0051u),
                                quintal_reg((hi >> 2) & 0x3333u, T[4], T[5], 0x0051u)};
        const uint32_t A1[4] = {quintal_reg((lo >> 16) & 0x3333u, T[2], T[3], 0x0040u),
                                quintal_reg((hi >> 16) & 0x3333u, T[6], T[7], 0x0040u),
                                quintal_reg((lo >> 18) & 0x3333u, T[2], T[3], 0x0051u),
                                quintal_reg((hi >> 18) & 0x3333u, T[6], T[7], 0x0051u)};
        mma_chunk(c0 + u, A0, A1);
      }
    }
  } else
  for (int c0 = c_begin; c0 < c_end; c0 += U) {
    uint2 wv[U];
#pragma unroll
    for (int u = 0; u < U; u++)
      if (c0 + u < c_end) wv[u] = ldg_stream_u2(codes + (size_t)(c0 + u) * 256);
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int c = c0 + u;
      if (c >= c_end) break;
      const uint8_t* s = ss + c * 32;
      const float sga = ue8m0_to_float(s[g]), sha = ue8m0_to_float(s[g + 8]);
      const float sgb = ue8m0_to_float(s[16 + g]), shb = ue8m0_to_float(s[24 + g]);
      const uint32_t lo = wv[u].x, hi = wv[u].y;
      const uint32_t lo2 = lo >> 2, hi2 = hi >> 2, lo16 = lo >> 16, hi16 = hi >> 16, lo18 = lo >> 18, hi18 = hi >> 18;
      uint32_t A0[4], A1[4];
      A0[0] = prmt(L, L, lo & 0x3333u);
      A0[1] = prmt(L, L, hi & 0x3333u);
      A0[2] = prmt(L, L, lo2 & 0x3333u);
      A0[3] = prmt(L, L, hi2 & 0x3333u);
      A1[0] = prmt(L, L, lo16 & 0x3333u);
      A1[1] = prmt(L, L, hi16 & 0x3333u);
      A1[2] = prmt(L, L, lo18 & 0x3333u);
      A1[3] = prmt(L, L, hi18 & 0x3333u);
#pragma unroll
      for (int nt = 0; nt < NT; nt++) {
        uint2 xa = make_uint2(0, 0), xb = make_uint2(0, 0);
        if (xr[nt] >= 0) {
          const uint8_t* xp = xbase + (size_t)xr[nt] * p.a_stride + (size_t)c * 64;
          xa = __ldg(reinterpret_cast<const uint2*>(xp));
          xb = __ldg(reinterpret_cast<const uint2*>(xp + 32));
        }
        float da[4] = {0.f, 0.f, 0.f, 0.f}, db[4] = {0.f, 0.f, 0.f, 0.f};
        mma_e4m3_16832(da, A0, xa.x, xa.y, da);
        mma_e4m3_16832(db, A1, xb.x, xb.y, db);
        const float as0 = sr0[nt] >= 0 ? ue8m0_to_float(__ldg(p.sA + (size_t)sr0[nt] * KC64 + c)) : 0.f;
        const float as1 = sr1[nt] >= 0 ? ue8m0_to_float(__ldg(p.sA + (size_t)sr1[nt] * KC64 + c)) : 0.f;
        acc[nt][0] = fmaf(fmaf(da[0], sga, db[0] * sgb), as0, acc[nt][0]);
        acc[nt][1] = fmaf(fmaf(da[1], sga, db[1] * sgb), as1, acc[nt][1]);
        acc[nt][2] = fmaf(fmaf(da[2], sha, db[2] * shb), as0, acc[nt][2]);
        acc[nt][3] = fmaf(fmaf(da[3], sha, db[3] * shb), as1, acc[nt][3]);
      }
    }
  }
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int j = nt * 8 + 2 * t + (i & 1);
      if (j >= nrows) continue;
      const int row = nb * 16 + g + ((i & 2) ? 8 : 0);
      w2_out_row(p, r0 + j)[row] = acc[nt][i];
    }
}

template <int NT>
__global__ void __launch_bounds__(128, NT == 1 ? 8 : 4) moe_w2_gemv_kernel(W2Args p) {
  moe_w2_gemv_body<NT>(p);
  if (p.ep_on) ep_publish(p.ep, ep_epoch(p.ep), 1);   // every CTA, including ones with no work
}


// out[t, :] = resid[t] (+ shared[t]) + sum_j w[t, j] * y[pos_of[t*k + j], :]  (fixed j order)
__global__ void moe_combine_kernel(const float* __restrict__ y, const int* __restrict__ pos_of,
                                   const float* __restrict__ wts, int k, int H,
                                   const __nv_bfloat16* __restrict__ resid,
                                   const __nv_bfloat16* __restrict__ shared_out,
                                   __nv_bfloat16* __restrict__ out, float* __restrict__ out_f32,
                                   int ar_on, ArDesc ar, int nsplit, long long split_stride,
                                   int ep_on, EpDesc ep) {
  pdl_entry();
  const int tok = blockIdx.x;
  const unsigned long long epoch = ar_on ? ar_epoch(ar) : 0ull;
  bool ep_ok = true;
  if (ep_on) ep_ok = ep_wait(ep, ep_epoch(ep), 1);     // every owner has returned this rank's rows
  __shared__ int pos[32];
  __shared__ float w[32];
  if (threadIdx.x < k) {
    pos[threadIdx.x] = !ep_ok ? -1 : pos_of ? pos_of[tok * k + threadIdx.x] : tok * k + threadIdx.x;
    w[threadIdx.x] = wts[tok * k + threadIdx.x];
  }
  __syncthreads();
  const int h_begin = blockIdx.y * 1024, h_end = min(H, h_begin + 1024);
  for (int h = h_begin + threadIdx.x * 4; h < h_end; h += blockDim.x * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < k; j++) {
      if (pos[j] < 0) continue;   // routed to an expert another rank owns
      float4 v = *reinterpret_cast<const float4*>(y + (size_t)pos[j] * H + h);
      for (int q = 1; q < nsplit; q++) {     // K-slice partials of the expert GEMV, slice order
        const float4 u = *reinterpret_cast<const float4*>(y + q * split_stride + (size_t)pos[j] * H + h);
        v.x += u.x; v.y += u.y; v.z += u.z; v.w += u.w;
      }
      acc.x = fmaf(w[j], v.x, acc.x); acc.y = fmaf(w[j], v.y, acc.y);
      acc.z = fmaf(w[j], v.z, acc.z); acc.w = fmaf(w[j], v.w, acc.w);
    }
    float r[4] = {acc.x, acc.y, acc.z, acc.w};
    if (ar_on) {   // expert combine -> all-reduce: push the partial (experts + shared) to every peer
      float4 v4 = acc;
      if (shared_out) {
        v4.x += __bfloat162float(shared_out[(size_t)tok * H + h]);
        v4.y += __bfloat162float(shared_out[(size_t)tok * H + h + 1]);
        v4.z += __bfloat162float(shared_out[(size_t)tok * H + h + 2]);
        v4.w += __bfloat162float(shared_out[(size_t)tok * H + h + 3]);
      }
      for (int q = 0; q < ar.world; q++)
        *reinterpret_cast<float4*>(ar_slot(ar, q, epoch, ar.rank) + (size_t)tok * H + h) = v4;
      continue;
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
      if (shared_out) r[i] += __bfloat162float(shared_out[(size_t)tok * H + h + i]);
      if (resid) r[i] += __bfloat162float(resid[(size_t)tok * H + h + i]);
      if (out) out[(size_t)tok * H + h + i] = __float2bfloat16(r[i]);
      if (out_f32) out_f32[(size_t)tok * H + h + i] = r[i];
    }
  }
  if (ar_on) ar_producer_arrive(ar, epoch);
  if (ep_on) {   // the return rows are consumed: the last CTA closes the layer's epoch
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      if (atomicAdd(ep.done, 1u) == gridDim.x * gridDim.y - 1) {
        *ep.done = 0u;
        *ep.ncall = *ep.ncall + 1ull;
        __threadfence();
      }
    }
  }
}

}  // namespace moet

using namespace moet;

void moe_w2_gemv(torch::Tensor a, torch::Tensor sa, c10::optional<torch::Tensor> gather, torch::Tensor pairs,
                 torch::Tensor n_pairs, torch::Tensor pool, int64_t codes_off, int64_t scale_off,
                 torch::Tensor slot_table, torch::Tensor out, int64_t N, int64_t K, int64_t rows_per_pair,
                 c10::optional<torch::Tensor> miss_count, c10::optional<torch::Tensor> pool8, int64_t codes_off8,
                 int64_t scale_off8, c10::optional<torch::Tensor> slot_table8, bool quintal,
                 c10::optional<torch::Tensor> ep, c10::optional<torch::Tensor> ret_rows) {
  TORCH_CHECK(K % 64 == 0 && N % 16 == 0, "moe_w2_gemv: N % 16, K % 64");
  TORCH_CHECK(a.stride(1) == 1 && a.size(1) == K, "moe_w2_gemv: A [rows, K] inner-contiguous");
  TORCH_CHECK(sa.is_contiguous() && sa.size(1) == K / 64, "moe_w2_gemv: sA [rows, K/64]");
  // out: [rows, N], or [ksplit, rows, N] K-slice partials (the consumers add the slices in order)
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.stride(-1) == 1, "moe_w2_gemv: out f32");
  const int ksplit = out.dim() == 3 ? out.size(0) : 1;
  TORCH_CHECK(pool.dim() == 2, "moe_w2_gemv: pool [slots, slot_bytes]");
  TORCH_CHECK(codes_off % 16 == 0 && scale_off % 16 == 0 && pool.stride(0) % 16 == 0, "moe_w2_gemv: alignment");
  W2Args p;
  p.A = (const uint8_t*)a.data_ptr(); p.sA = (const uint8_t*)sa.data_ptr(); p.a_stride = a.stride(0);
  p.gather = gather.has_value() && gather->defined() ? gather->data_ptr<int>() : nullptr;
  p.pairs = (const int4*)pairs.data_ptr<int>(); p.n_pairs = n_pairs.data_ptr<int>();
  p.pool = (const uint8_t*)pool.data_ptr(); p.slot_bytes = pool.stride(0);
  p.codes_off = codes_off; p.scale_off = scale_off;
  p.slot_table = slot_table.data_ptr<int>();
  p.out = out.data_ptr<float>(); p.out_stride = out.stride(-2);
  p.part_stride = out.dim() == 3 ? out.stride(0) : 0;
  p.cps = (int)((K / 64 + ksplit - 1) / ksplit);
  p.N = N; p.K = K;
  p.miss_count = miss_count.has_value() && miss_count->defined() ? miss_count->data_ptr<int>() : nullptr;
  p.pool8 = nullptr; p.slot_table8 = nullptr; p.slot_bytes8 = p.codes_off8 = p.scale_off8 = 0;
  p.quintal = 0;
  if (pool8.has_value() && pool8->defined()) {
    TORCH_CHECK(slot_table8.has_value() && pool8->dim() == 2 && pool8->stride(0) % 16 == 0 && codes_off8 % 16 == 0 &&
                scale_off8 % 16 == 0, "moe_w2_gemv: delta pool [slots, bytes] with a slot table, 16-byte aligned");
    p.pool8 = (const uint8_t*)pool8->data_ptr(); p.slot_bytes8 = pool8->stride(0);
    p.codes_off8 = codes_off8; p.scale_off8 = scale_off8; p.slot_table8 = slot_table8->data_ptr<int>();
    p.quintal = quintal ? 1 : 0;
    TORCH_CHECK(!quintal || codes_off8 % 8 == 0, "moe_w2_gemv: quintal plane offset");
  }
  p.ep_on = ep.has_value() && ep->defined();
  p.ret_rows = nullptr; p.ep = EpDesc{};
  if (p.ep_on) {
    p.ep = ep_desc_from(*ep);
    TORCH_CHECK(ret_rows.has_value() && ret_rows->defined() && N == p.ep.H,
                "moe_w2_gemv: the EP return leg needs ret_rows and N == H");
    p.ret_rows = ret_rows->data_ptr<int>();
  }
  const int max_pairs = pairs.size(0);
  const int wpc = 4;
  TORCH_CHECK(!p.ep_on || ksplit == 1, "moe_w2_gemv: the EP return leg takes no K slices");
  dim3 grid((N / 16 + wpc - 1) / wpc, max_pairs, ksplit);
  auto stream = at::cuda::getCurrentCUDAStream();
  // scale stage per warp; split FP4 adds a 640-entry u16 digit table per warp
  const size_t smem = (size_t)wpc * 16 * (K / 32) + (p.quintal ? (size_t)wpc * 640 * 2 : 0);
  TORCH_CHECK(smem <= 48 * 1024, "moe_w2_gemv: K too large for the shared scale stage");
  switch (rows_per_pair) {
    case 8: launch_k(moe_w2_gemv_kernel<1>, grid, wpc * 32, smem, stream, p); break;
    case 16: launch_k(moe_w2_gemv_kernel<2>, grid, wpc * 32, smem, stream, p); break;
    case 32: launch_k(moe_w2_gemv_kernel<4>, grid, wpc * 32, smem, stream, p); break;
    default: TORCH_CHECK(false, "moe_w2_gemv: rows_per_pair must be 8/16/32");
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void moe_combine(torch::Tensor y, torch::Tensor pos_of, torch::Tensor wts, c10::optional<torch::Tensor> resid,
                 c10::optional<torch::Tensor> shared_out, c10::optional<torch::Tensor> out,
                 c10::optional<torch::Tensor> out_f32, c10::optional<torch::Tensor> ar,
                 c10::optional<torch::Tensor> ep) {
  // y: [R, H] or [nsplit, R, H] (K-slice partials, summed in slice order); pos_of may be
  // empty (identity: row t * k + j); ep: wait for the owners' returns first
  const int ep_on = ep.has_value() && ep->defined();
  EpDesc ed{};
  if (ep_on) ed = ep_desc_from(*ep);
  const int T = wts.size(0), k = wts.size(1), H = y.size(-1);
  const int nsplit = y.dim() == 3 ? y.size(0) : 1;
  const long long split_stride = y.dim() == 3 ? y.stride(0) : 0;
  TORCH_CHECK(y.stride(-1) == 1 && y.stride(-2) == H, "moe_combine: y rows contiguous");
  const int ar_on = ar.has_value() && ar->defined();
  ArDesc d{};
  if (ar_on) {
    d = ar_desc_from(*ar);
    TORCH_CHECK(!resid.has_value() || !resid->defined(), "moe_combine: the all-reduce push takes no residual");
    TORCH_CHECK((int64_t)T * H <= d.cap, "moe_combine: T*H exceeds the all-reduce slot");
  }
  TORCH_CHECK(H % 4 == 0 && k <= 32, "moe_combine: H % 4, k <= 32");
  if (T == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_k(moe_combine_kernel, dim3(T, (H + 1023) / 1024), 256, 0, stream, y.data_ptr<float>(),
           pos_of.numel() ? pos_of.data_ptr<int>() : nullptr, wts.data_ptr<float>(), k, H,
                                            (const __nv_bfloat16*)opt_ptr(resid), (const __nv_bfloat16*)opt_ptr(shared_out),
                                            (__nv_bfloat16*)opt_ptr(out), (float*)opt_ptr(out_f32), ar_on, d,
                                            nsplit, split_stride, ep_on, ed);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
