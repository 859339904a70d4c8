// tcgen05 block-scaled "swap-AB" GEMM: out[tok, row] = sum_k act[tok, k] * W[row, k]
// with the weights as the M = 128 operand and up to NT <= 128 tokens as N.
//
//   ASRC = 0: W is a 2-bit codebook expert (fragment-major code + UE8M0 scale
//             planes in a slot pool); work items are expert pairs (e, rows).
//             The 2-bit codes are decoded to e4m3 {-4,-1,1,4} straight into
//             the SMEM operand tile; block scales go to TMEM unchanged.
//   ASRC = 1: W is dense e4m3 row-major with UE8M0 128x128 block scales;
//             work items are token tiles.
// Activations are e4m3 with UE8M0 per-64 scales.  For ASRC = 0 they are in the
// w2 layout, whose in-k32 permutation equals the order the decode writes A in,
// so A and B agree on the physical k order (the MMA sums over k).
//
// Pipeline: K in stages of 128 (4 MMAs of K = 32), 3 SMEM buffers.  All 128
// threads stage a buffer (A decode/copy, B rows, scale-factor atoms), then one
// thread copies the scale factors into TMEM, issues the 4 MMAs and commits to
// the buffer's mbarrier; threads wait on that mbarrier (bounded) before
// restaging the buffer three stages later.  Accumulators stay in TMEM until the
// epilogue reads them with tcgen05.ld (warp w owns rows 32w..32w+31).
#include "tcgen05.cuh"
#include "torch_glue.h"

namespace moet {

struct TcArgs {
  // activations (B operand)
  const uint8_t* act; const uint8_t* act_s; long long act_stride; int act_groups;   // act_s: [rows, K/64]
  const int* gather;                        // sorted row -> activation row (experts), may be null
  // expert source (ASRC 0)
  const int4* pairs; const int* n_pairs;
  const uint8_t* pool; long long slot_bytes; long long codes_off, scale_off; const int* slot_table;
  // dense source (ASRC 1)
  const uint8_t* W; const uint8_t* sW; int sw_cols;
  int T;                                    // tokens (dense)
  // output
  void* out; long long out_stride; int out_f32; const __nv_bfloat16* resid;
  int N, K;
  int* miss_count; int* status;
  int dbg;                                  // profiling switches (0 in production)
};

constexpr int kStageK = 128;
constexpr int kBufs = 3;

template <int NT>
struct TcSmem {
  static constexpr int A = 128 * kStageK;       // 16 KB
  static constexpr int B = NT * kStageK;        // NT * 128 B
  static constexpr int SF = 512;
  static constexpr int STAGE = A + B + 2 * SF;
  static constexpr int TOTAL = kBufs * STAGE;
  static constexpr int TMEM_COLS = NT + 8 * kBufs <= 32 ? 32 : (NT + 8 * kBufs <= 64 ? 64 : (NT + 8 * kBufs <= 128 ? 128 : 256));
};

template <int NT, int ASRC>
__global__ void __launch_bounds__(128) tc_gemm_kernel(TcArgs p) {
  extern __shared__ __align__(1024) uint8_t sm[];
  __shared__ uint64_t bars[kBufs + 2];   // stage buffers, accumulator done, drain
  __shared__ uint32_t taddr_s;
  using L = TcSmem<NT>;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int m0 = blockIdx.x * 128;
  if (m0 >= p.N) return;
  int r0 = 0, nrows = 0;
  const uint8_t* codes = nullptr; const uint8_t* wsc = nullptr;
  if constexpr (ASRC == 0) {
    const int pi = blockIdx.y;
    if (pi >= *p.n_pairs) return;
    const int4 pr = p.pairs[pi];
    r0 = pr.y; nrows = pr.z;
    const int slot = p.slot_table[pr.x];
    if (slot < 0) {
      if (blockIdx.x == 0 && tid == 0 && p.miss_count) atomicAdd(p.miss_count, 1);
      for (int i = tid; i < nrows * 128; i += 128) {
        const int n = i / 128, row = m0 + i % 128;
        if (row < p.N) reinterpret_cast<float*>(p.out)[(size_t)(r0 + n) * p.out_stride + row] = 0.f;
      }
      return;
    }
    const uint8_t* base = p.pool + (size_t)slot * p.slot_bytes;
    codes = base + p.codes_off;
    wsc = base + p.scale_off;
  } else {
    r0 = blockIdx.y * NT;
    if (r0 >= p.T) return;
    nrows = min(NT, p.T - r0);
  }
  const int K = p.K, KC = K / 64, KS = K / 32;
  const int nstages = K / kStageK;

  if (warp == 0) tc::tmem_alloc(&taddr_s, L::TMEM_COLS);
  if (tid == 0) { for (int i = 0; i <= kBufs + 1; i++) tc::mbar_init(&bars[i], 1); }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = taddr_s;

  // B rows handled by this thread: (n, 16-byte piece c) for i = tid, tid+128, ...
  // activation row of token column n
  auto act_row = [&](int n) -> int {
    if (n >= nrows) return -1;
    const int r = r0 + n;
    return p.gather ? __ldg(p.gather + r) : r;
  };

  // Each thread keeps the next stage's global data in registers (loaded one
  // stage ahead) so staging a buffer never waits on a global round trip.
  constexpr int BPT = (NT * 8 + 127) / 128;          // 16-byte B pieces per thread
  uint2 cw[4];                                       // 2-bit codes (ASRC 0)
  uint4 wv[8];                                       // dense rows (ASRC 1)
  uint4 bv[BPT];
  uint32_t sfa_v = 0, sfb_v = 0;
  auto load_stage = [&](int s) {
    if (p.dbg & 1) return;
    if constexpr (ASRC == 0) {
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int nb = (m0 >> 4) + 2 * warp + (i >> 1), kb = 2 * s + (i & 1);
        cw[i] = ldg_stream_u2(codes + ((size_t)(nb * KC + kb) * 32 + lane) * 8);
      }
      const int m = tid, nb = (m0 >> 4) + (m >> 4), r = m & 15;
      const uint8_t* sp = wsc + ((size_t)nb * KS + 4 * s) * 16 + r;
      sfa_v = (uint32_t)__ldg(sp) | ((uint32_t)__ldg(sp + 16) << 8) | ((uint32_t)__ldg(sp + 32) << 16) |
              ((uint32_t)__ldg(sp + 48) << 24);
    } else {
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int i = tid + 128 * j;
        const int row = (i & 7) + 8 * (i >> 6), c = (i >> 3) & 7;
        const int grow = min(m0 + row, p.N - 1);
        wv[j] = ldg_stream_u4(p.W + (size_t)grow * K + (size_t)s * kStageK + c * 16);
      }
      sfa_v = (uint32_t)__ldg(p.sW + (size_t)(m0 >> 7) * p.sw_cols + s) * 0x01010101u;
    }
#pragma unroll
    for (int j = 0; j < BPT; j++) {
      const int i = tid + 128 * j;
      bv[j] = make_uint4(0, 0, 0, 0);
      if (i < NT * 8) {
        const int n = (i & 7) + 8 * (i >> 6), c = (i >> 3) & 7;
        const int ar = act_row(n);
        if (ar >= 0) bv[j] = __ldg(reinterpret_cast<const uint4*>(p.act + (size_t)ar * p.act_stride + (size_t)s * kStageK + c * 16));
      }
    }
    if (tid < NT) {
      const int ar = act_row(tid);
      sfb_v = 0;
      if (ar >= 0) {
        const uint32_t a0 = __ldg(p.act_s + (size_t)ar * p.act_groups + 2 * s);
        const uint32_t a1 = __ldg(p.act_s + (size_t)ar * p.act_groups + 2 * s + 1);
        sfb_v = a0 | (a0 << 8) | (a1 << 16) | (a1 << 24);
      }
    }
  };
  load_stage(0);

  bool ok = true;
  for (int s = 0; s < nstages && ok; s++) {
    const int buf = s % kBufs;
    uint8_t* sA = sm + buf * L::STAGE;
    uint8_t* sB = sA + L::A;
    uint8_t* sSFA = sB + L::B;
    uint8_t* sSFB = sSFA + L::SF;
    if (s >= kBufs) {
      if (!tc::mbar_wait(&bars[buf], ((s / kBufs) - 1) & 1)) { ok = false; }
      if (!__syncthreads_and(ok)) { ok = false; break; }
      tc::fence_after();
    }
    // ---- stage registers -> shared memory ----
    if (p.dbg & 4) {} else if constexpr (ASRC == 0) {
      constexpr uint32_t LUT = 0x4838B8C8u;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int rb = 2 * warp + (i >> 1);           // row block inside the tile
        const int kloc = (i & 1) * 64;                // chunk offset inside the stage
        const uint32_t lo = cw[i].x, hi = cw[i].y;
        const uint2 ra = make_uint2(prmt(LUT, LUT, lo & 0x3333u), prmt(LUT, LUT, (lo >> 2) & 0x3333u));
        const uint2 rb2 = make_uint2(prmt(LUT, LUT, (lo >> 16) & 0x3333u), prmt(LUT, LUT, (lo >> 18) & 0x3333u));
        const uint2 ha = make_uint2(prmt(LUT, LUT, hi & 0x3333u), prmt(LUT, LUT, (hi >> 2) & 0x3333u));
        const uint2 hb = make_uint2(prmt(LUT, LUT, (hi >> 16) & 0x3333u), prmt(LUT, LUT, (hi >> 18) & 0x3333u));
        const int row0 = rb * 16 + g, row1 = row0 + 8;
        *reinterpret_cast<uint2*>(sA + tc::kmajor_off(row0, kloc + 8 * t, kStageK)) = ra;
        *reinterpret_cast<uint2*>(sA + tc::kmajor_off(row0, kloc + 32 + 8 * t, kStageK)) = rb2;
        *reinterpret_cast<uint2*>(sA + tc::kmajor_off(row1, kloc + 8 * t, kStageK)) = ha;
        *reinterpret_cast<uint2*>(sA + tc::kmajor_off(row1, kloc + 32 + 8 * t, kStageK)) = hb;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int i = tid + 128 * j;
        const int row = (i & 7) + 8 * (i >> 6), c = (i >> 3) & 7;
        *reinterpret_cast<uint4*>(sA + tc::kmajor_off(row, c * 16, kStageK)) = wv[j];
      }
    }
    *reinterpret_cast<uint32_t*>(sSFA + (tid & 31) * 16 + (tid >> 5) * 4) = sfa_v;
#pragma unroll
    for (int j = 0; j < BPT; j++) {
      const int i = tid + 128 * j;
      if (i < NT * 8) {
        const int n = (i & 7) + 8 * (i >> 6), c = (i >> 3) & 7;
        *reinterpret_cast<uint4*>(sB + tc::kmajor_off(n, c * 16, kStageK)) = bv[j];
      }
    }
    if (tid < NT) *reinterpret_cast<uint32_t*>(sSFB + (tid & 31) * 16 + (tid >> 5) * 4) = sfb_v;
    if (s + 1 < nstages) load_stage(s + 1);
    tc::fence_proxy_async_smem();
    tc::fence_before();
    __syncthreads();
    if (tid == 0 && (p.dbg & 2)) { tc::commit(&bars[buf]); if (s == nstages - 1) tc::commit(&bars[kBufs]); }
    if (tid == 0 && !(p.dbg & 2)) {
      tc::fence_after();
      const uint32_t t_sfa = tmem + NT + 8 * buf, t_sfb = t_sfa + 4;
      tc::cp_sf_32x128b_warpx4(t_sfa, tc::smem_desc(tc::smem_addr(sSFA), 0, 128));
      tc::cp_sf_32x128b_warpx4(t_sfb, tc::smem_desc(tc::smem_addr(sSFB), 0, 128));
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {
        const uint64_t da = tc::smem_desc(tc::smem_addr(sA + kk * 256), 128, 1024);
        const uint64_t db = tc::smem_desc(tc::smem_addr(sB + kk * 256), 128, 1024);
        tc::mma_mxf8(tmem, da, db, tc::idesc_mxf8(128, NT, kk, kk), (s > 0 || kk > 0) ? 1u : 0u, t_sfa, t_sfb);
      }
      tc::commit(&bars[buf]);
      if (s == nstages - 1) tc::commit(&bars[kBufs]);
    }
  }
  if (ok) ok = tc::mbar_wait(&bars[kBufs], 0);
  if (!__syncthreads_and(ok)) {
    if (tid == 0) {
      set_status(p.status, kTimeout);
      // drain: a commit tracks every MMA this thread issued; wait (bounded) before TMEM is freed
      tc::commit(&bars[kBufs + 1]);
      tc::mbar_wait(&bars[kBufs + 1], 0);
    }
  } else {
    tc::fence_after();
    const int row = warp * 32 + lane;
    const int grow = m0 + row;
#pragma unroll 1
    for (int c0 = 0; c0 < NT; c0 += 8) {
      uint32_t r[8];
      tc::tmem_ld8(tmem + ((uint32_t)(warp * 32) << 16) + c0, r);
      tc::tmem_wait_ld();
      if (grow < p.N) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const int n = c0 + j;
          if (n >= nrows) break;
          const size_t off = (size_t)(r0 + n) * p.out_stride + grow;
          float v = __uint_as_float(r[j]);
          if (p.resid) v += __bfloat162float(p.resid[off]);
          if (p.out_f32) reinterpret_cast<float*>(p.out)[off] = v;
          else reinterpret_cast<__nv_bfloat16*>(p.out)[off] = __float2bfloat16(v);
        }
      }
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) { tc::tmem_dealloc(tmem, L::TMEM_COLS); tc::tmem_relinquish(); }
}

template <int NT, int ASRC>
static void launch_tc(const TcArgs& a, dim3 grid, cudaStream_t stream) {
  using L = TcSmem<NT>;
  moet_allow_max_smem(tc_gemm_kernel<NT, ASRC>);
  // ask for the full shared-memory carveout so several CTAs share an SM
  cudaFuncSetAttribute(tc_gemm_kernel<NT, ASRC>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  tc_gemm_kernel<NT, ASRC><<<grid, 128, L::TOTAL, stream>>>(a);
}

template <int ASRC>
static void dispatch_tc(int nt, const TcArgs& a, dim3 grid, cudaStream_t stream) {
  switch (nt) {
    case 8: launch_tc<8, ASRC>(a, grid, stream); break;
    case 16: launch_tc<16, ASRC>(a, grid, stream); break;
    case 32: launch_tc<32, ASRC>(a, grid, stream); break;
    case 64: launch_tc<64, ASRC>(a, grid, stream); break;
    case 128: launch_tc<128, ASRC>(a, grid, stream); break;
    default: TORCH_CHECK(false, "tc gemm: token tile must be 8/16/32/64/128");
  }
}

}  // namespace moet

using namespace moet;

// Expert GEMM over the pair list (2-bit planes), tokens per pair = nt.
void tc_moe_w2(torch::Tensor a, torch::Tensor sa, c10::optional<torch::Tensor> gather, torch::Tensor pairs,
               torch::Tensor n_pairs, torch::Tensor pool, int64_t codes_off, int64_t scale_off,
               torch::Tensor slot_table, torch::Tensor out, int64_t N, int64_t K, int64_t nt,
               c10::optional<torch::Tensor> miss_count, torch::Tensor status, int64_t dbg) {
  TORCH_CHECK(K % kStageK == 0 && N % 128 == 0, "tc_moe_w2: K % 128, N % 128");
  TORCH_CHECK(a.stride(1) == 1 && a.size(1) == K && a.stride(0) % 16 == 0, "tc_moe_w2: activations");
  TORCH_CHECK(out.scalar_type() == at::kFloat, "tc_moe_w2: f32 out");
  TcArgs p{};
  p.act = (const uint8_t*)a.data_ptr(); p.act_s = (const uint8_t*)sa.data_ptr(); p.act_stride = a.stride(0);
  p.act_groups = sa.size(1);
  p.gather = gather.has_value() && gather->defined() ? gather->data_ptr<int>() : nullptr;
  p.pairs = (const int4*)pairs.data_ptr<int>(); p.n_pairs = n_pairs.data_ptr<int>();
  p.pool = (const uint8_t*)pool.data_ptr(); p.slot_bytes = pool.stride(0); p.codes_off = codes_off; p.scale_off = scale_off;
  p.slot_table = slot_table.data_ptr<int>();
  p.out = out.data_ptr(); p.out_stride = out.stride(0); p.out_f32 = 1;
  p.N = N; p.K = K;
  p.miss_count = miss_count.has_value() && miss_count->defined() ? miss_count->data_ptr<int>() : nullptr;
  p.status = status.data_ptr<int>();
  p.dbg = (int)dbg;
  dim3 grid((N + 127) / 128, pairs.size(0));
  dispatch_tc<0>((int)nt, p, grid, at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Dense FP8 GEMM: out[T, N] (+ resid) = a[T, K] * w[N, K]^T
void tc_gemm_fp8(torch::Tensor a, torch::Tensor sa, torch::Tensor w, torch::Tensor sw, torch::Tensor out,
                 c10::optional<torch::Tensor> resid, int64_t nt, torch::Tensor status) {
  const int T = a.size(0), K = a.size(1), N = w.size(0);
  TORCH_CHECK(K % kStageK == 0 && w.size(1) == K && w.is_contiguous(), "tc_gemm_fp8: K % 128, contiguous W");
  TORCH_CHECK(a.stride(1) == 1 && a.stride(0) % 16 == 0 && sa.size(1) == K / 64, "tc_gemm_fp8: activations");
  TORCH_CHECK(sw.size(0) == (N + 127) / 128 && sw.size(1) == K / 128, "tc_gemm_fp8: weight scales");
  if (T == 0) return;
  TcArgs p{};
  p.act = (const uint8_t*)a.data_ptr(); p.act_s = (const uint8_t*)sa.data_ptr(); p.act_stride = a.stride(0);
  p.act_groups = sa.stride(0);
  p.W = (const uint8_t*)w.data_ptr(); p.sW = (const uint8_t*)sw.data_ptr(); p.sw_cols = sw.size(1);
  p.T = T;
  p.out = out.data_ptr(); p.out_stride = out.stride(0); p.out_f32 = out.scalar_type() == at::kFloat;
  p.resid = resid.has_value() && resid->defined() ? (const __nv_bfloat16*)resid->data_ptr() : nullptr;
  if (p.resid) TORCH_CHECK(resid->stride(0) == out.stride(0), "tc_gemm_fp8: resid layout");
  p.N = N; p.K = K; p.status = status.data_ptr<int>();
  dim3 grid((N + 127) / 128, (T + nt - 1) / nt);
  dispatch_tc<1>((int)nt, p, grid, at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
