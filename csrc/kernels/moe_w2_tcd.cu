// 2-bit codebook expert GEMV for decode on the 5th-generation tensor cores.
//
//   out[s][row_r, n] = sum_{k in slice s} A[row_r, k] * W_e[n, k]   for every pair (e, rows)
//
// Decode routes a handful of tokens to each expert, so the MMA's N is the pair's token
// rows (8 or 16) and M = 128 weight rows.  Instead of mma.sync fragments with per-k32
// scale arithmetic (moe_w2.cu), this kernel hands the block scales to the tensor core:
//   * every thread fetches (cp.async, a 5-stage ring per CTA, three stages ahead) the
//     32 code bytes it will decode itself -- 8 rows-of-16 x 64 k of one row pair -- and
//     writes 128 e4m3 weights (one prmt per four codes) into the K-major A tile, so no
//     thread waits for another thread's loads;
//   * the UE8M0 block-32 weight scales (raw plane bytes) and the activations' per-64
//     scales become the MMA's scale-factor atoms and go to TMEM with tcgen05.cp; the
//     block-scaled kind::mxf8f6f4 MMA applies them, so no scale arithmetic is issued;
//   * the activation rows are copied by cp.async straight into the K-major B layout;
//   * one thread issues four MMAs (K = 32 each) per 128-K stage and commits to the
//     stage's mbarrier; the A tile is double-buffered.
// Work = (pair, 128-row tile, K slice) tasks in contiguous ranges per CTA; slice s
// writes out[s] and the consumers (swiglu_quant / moe_combine) add slices in order.
// Missing experts (slot < 0) produce zero rows and count a miss.  Every wait is
// bounded; a timeout records kTimeout, drains the MMAs in flight and frees TMEM.
//
// Measured on B200 (DS4 decode shape, 24 routed pairs of one token, w13 N = 3072,
// K = 4096, 85 MB): 183 us at one CTA per SM and 210 us at three, against 53 us for the
// mma.sync GEMV.  With 8 token columns each 128-k stage waits on the MMA issue-to-commit
// round trip, and more CTAs per SM do not add throughput; the runner therefore keeps the
// mma.sync GEMV for decode and this kernel is opt-in (MOET_W2_DECODE=tcd).
#include "tcgen05.cuh"
#include "torch_glue.h"

namespace moet {
namespace tcd {

constexpr int kThreads = 128;
constexpr int kAhead = 3;         // cp.async prefetch distance (stages)
constexpr int kA = 16384;         // 128 rows x 128 k e4m3
constexpr int kCodes = 4096, kSfRaw = 512;

// NA A-tile buffers: stage j waits for the MMAs of stage j - NA; the ring holds NA + kAhead stages
template <int NT, int NA>
struct Cfg {
  static constexpr int B = NT * 128;
  static constexpr int SFB = 16 * ((NT * 4 + 15) / 16);
  static constexpr int RING = (kCodes + kSfRaw + B + SFB + 127) / 128 * 128;     // one ring stage
  static constexpr int NR = NA + kAhead;
  static constexpr int SMEM = NR * RING + NA * kA + NA * 1024 + 1024;   // + SF atoms, alignment slack
};

MOET_DEVICE void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
MOET_DEVICE void cp_async4(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
MOET_DEVICE void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
MOET_DEVICE void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

}  // namespace tcd

struct TcdArgs {
  const uint8_t* A; const uint8_t* sA; long long a_stride;   // activations (w2 layout), per-64 scales
  const int* gather;                                         // sorted row -> activation row (null: identity)
  const int4* pairs; const int* n_pairs;
  const uint8_t* pool; long long slot_bytes, codes_off, scale_off;
  const int* slot_table;
  float* out; long long out_stride, part_stride;
  int N, K, ksplit, spt;        // K slices, 128-k stages per slice
  int* miss_count; int* status;
};

template <int NT, int NA>
__global__ void __launch_bounds__(tcd::kThreads, 1) moe_w2_tcd_kernel(TcdArgs p) {
  using namespace tcd;
  using Cf = Cfg<NT, NA>;
  constexpr int kRing = Cf::NR;
  extern __shared__ uint8_t tcd_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tcd_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = sm;                                   // kRing x [codes | sf raw | B | sfb raw]
  uint8_t* abuf = ring + kRing * Cf::RING;              // NA x A tile
  uint8_t* atoms = abuf + NA * kA;                      // NA x [SFA 512 | SFB 512]
  __shared__ uint64_t mma_done[NA], drain;
  __shared__ uint32_t taddr_s;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int i = 0; i < NA; i++) tc::mbar_init(&mma_done[i], 1);
    tc::mbar_init(&drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tc::tmem_alloc(&taddr_s, 64);     // accumulator cols [0, 16), SF cols 16 + 8 b
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = taddr_s;
  pdl_entry();

  const int KC = p.K >> 6, KS = p.K >> 5, nstg = p.K >> 7;
  const int NRT = (p.N + 127) >> 7;
  const int ntasks = *p.n_pairs * p.ksplit * NRT;
  const int per = (ntasks + (int)gridDim.x - 1) / (int)gridDim.x;
  const int tb = (int)blockIdx.x * per, te = min(ntasks, tb + per);
  const int nstages = te > tb ? (te - tb) * p.spt : 0;

  // Stage cursor: task order pair (slowest), slice, row tile; spt stages per task.  Advanced
  // one stage at a time (no divisions in the loop); caches the pair and its slot.
  struct Cursor {
    int pi, sl, rt, l;
    int4 pr; int slot;
  };
  auto cur_init = [&](Cursor& c) {
    c.rt = tb % NRT;
    const int r = tb / NRT;
    c.sl = r % p.ksplit; c.pi = r / p.ksplit; c.l = 0;
    c.pr = make_int4(0, 0, 0, 0); c.slot = -1;
    if (tb < te) { c.pr = p.pairs[c.pi]; c.slot = p.slot_table[c.pr.x]; }
  };
  auto cur_next = [&](Cursor& c, bool load) {
    if (++c.l < p.spt) return;
    c.l = 0;
    if (++c.rt < NRT) return;
    c.rt = 0;
    if (++c.sl < p.ksplit) return;
    c.sl = 0; c.pi++;
    if (load) { c.pr = p.pairs[c.pi]; c.slot = p.slot_table[c.pr.x]; }
  };
  // issue the cp.async group of the stage under cursor c into ring slot j % kRing (always commits a group)
  auto issue = [&](int j, const Cursor& c) {
    if (j < nstages) {
      const int4 pr = c.pr;
      const int slot = c.slot;
      const int g = c.sl * p.spt + c.l;
      const bool valid = g < nstg;
      uint8_t* rs = ring + (j % kRing) * Cf::RING;
      const uint32_t rsa = tc::smem_addr(rs);
      const bool live = slot >= 0 && valid;
      const uint8_t* base = p.pool + (size_t)(slot < 0 ? 0 : slot) * p.slot_bytes;
      const int stg = valid ? g : 0;
      {   // codes: thread = (row block, 64-k chunk, row pair) unit of 32 bytes
        const int rb = tid >> 4, kl = (tid >> 3) & 1, lp = tid & 7;
        const int nb = c.rt * 8 + rb;
        const bool ok = live && nb * 16 < p.N;
        const uint8_t* src = base + p.codes_off + ((size_t)nb * KC + 2 * stg + kl) * 256 + lp * 32;
        tcd::cp_async16(rsa + tid * 32, ok ? src : p.pool, ok ? 16 : 0);
        tcd::cp_async16(rsa + tid * 32 + 16, ok ? src + 16 : p.pool, ok ? 16 : 0);
      }
      if (tid < 32) {   // raw scale bytes: (row block, k32 block) -> 16 rows
        const int rb = tid >> 2, kb = tid & 3;
        const int nb = c.rt * 8 + rb;
        const bool ok = live && nb * 16 < p.N;
        const uint8_t* src = base + p.scale_off + ((size_t)nb * KS + 4 * stg + kb) * 16;
        tcd::cp_async16(rsa + kCodes + tid * 16, ok ? src : p.pool, ok ? 16 : 0);
      }
      if (tid < NT * 8) {   // activation rows into the K-major B layout
        const int n = tid >> 3, c16 = tid & 7;
        const bool ok = valid && n < pr.z;
        const int row = ok ? (p.gather ? __ldg(p.gather + pr.y + n) : pr.y + n) : 0;
        const uint8_t* src = p.A + (size_t)row * p.a_stride + (size_t)stg * 128 + c16 * 16;
        tcd::cp_async16(rsa + kCodes + kSfRaw + tc::kmajor_off(n, c16 * 16, 128), ok ? src : p.A, ok ? 16 : 0);
      }
      if (tid < NT) {       // activation scales: the aligned word holding groups 2 stg, 2 stg + 1
        const bool ok = valid && tid < pr.z;
        const int row = ok ? (p.gather ? __ldg(p.gather + pr.y + tid) : pr.y + tid) : 0;
        const size_t off = ((size_t)row * KC + 2 * stg) & ~size_t(3);
        tcd::cp_async4(rsa + kCodes + kSfRaw + Cf::B + tid * 4, ok ? p.sA + off : p.sA, ok ? 4 : 0);
      }
    }
    tcd::cp_commit();
  };

  bool ok = true;
  Cursor ci, cc;            // issue cursor (kAhead stages ahead), consume cursor
  cur_init(ci);
  cur_init(cc);
  for (int j = 0; j < kAhead; j++) {
    issue(j, ci);
    if (j < nstages) cur_next(ci, j + 1 < nstages);
  }
  uint32_t uses[NA];
#pragma unroll
  for (int i = 0; i < NA; i++) uses[i] = 0u;
  constexpr uint32_t LUT = 0x4838B8C8u;   // e4m3 {-4, -1, +1, +4}
  for (int j = 0; j < nstages && ok; j++) {
    const int b = j % NA;
    if (uses[b] > 0) {      // the MMAs of stage j - NA have released A buffer b and their ring slot
      const bool w = tc::mbar_wait(&mma_done[b], (uses[b] - 1) & 1);
      if (!__syncthreads_and(w)) { ok = false; break; }
    }
    issue(j + kAhead, ci);
    if (j + kAhead < nstages) cur_next(ci, j + kAhead + 1 < nstages);
    tcd::cp_wait<kAhead>();
    const int4 pr = cc.pr;
    const int g_stage = cc.sl * p.spt + cc.l;
    const uint8_t* rs = ring + (j % kRing) * Cf::RING;
    uint8_t* A = abuf + b * kA;
    uint8_t* sfa = atoms + b * 1024;
    uint8_t* sfb = sfa + 512;
    {   // 32 code bytes -> 128 e4m3 weights of rows (g, g + 8), 64 k
      const int rb = tid >> 4, kl = (tid >> 3) & 1, g = tid & 7;
      const uint4 c0 = *reinterpret_cast<const uint4*>(rs + tid * 32);
      const uint4 c1 = *reinterpret_cast<const uint4*>(rs + tid * 32 + 16);
      const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};   // lane t: (w[2t] row g, w[2t+1] row g+8)
      uint32_t ra[2][8], rbv[2][8];   // [row half][t*2 + {0,1}]: k32a / k32b bytes
#pragma unroll
      for (int t = 0; t < 4; t++)
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const uint32_t x = w[2 * t + h];
          const uint32_t m = x & 0x33333333u, q = (x >> 2) & 0x33333333u;
          ra[h][2 * t] = prmt(LUT, LUT, m);
          ra[h][2 * t + 1] = prmt(LUT, LUT, q);
          rbv[h][2 * t] = prmt(LUT, LUT, m >> 16);
          rbv[h][2 * t + 1] = prmt(LUT, LUT, q >> 16);
        }
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int m = rb * 16 + g + 8 * h;
        uint8_t* dst = A + tc::kmajor_off(m, kl * 64, 128);
        // k16 chunks of the 64-k half: [t0,t1] k32a, [t2,t3] k32a, [t0,t1] k32b, [t2,t3] k32b
        *reinterpret_cast<uint4*>(dst) = make_uint4(ra[h][0], ra[h][1], ra[h][2], ra[h][3]);
        *reinterpret_cast<uint4*>(dst + 128) = make_uint4(ra[h][4], ra[h][5], ra[h][6], ra[h][7]);
        *reinterpret_cast<uint4*>(dst + 256) = make_uint4(rbv[h][0], rbv[h][1], rbv[h][2], rbv[h][3]);
        *reinterpret_cast<uint4*>(dst + 384) = make_uint4(rbv[h][4], rbv[h][5], rbv[h][6], rbv[h][7]);
      }
    }
    if (tid < 32) {   // weight scales: raw [row block][k32 block][16 rows] -> SF atom (row m, k block kb)
      const int rbk = tid >> 2, kb = tid & 3;
      const uint4 v = *reinterpret_cast<const uint4*>(rs + kCodes + tid * 16);
      const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const int m = rbk * 16 + i;
        sfa[(m & 31) * 16 + (m >> 5) * 4 + kb] = (uint8_t)(wv[i >> 2] >> ((i & 3) * 8));
      }
    }
    if (tid < 32) {   // activation scales: token rows 0..31 of the atom (NT rows used)
      uint32_t v = 0;
      if (tid < NT) {
        const uint32_t wd = *reinterpret_cast<const uint32_t*>(rs + kCodes + kSfRaw + Cf::B + tid * 4);
        if (tid < pr.z) {
          const int row = p.gather ? __ldg(p.gather + pr.y + tid) : pr.y + tid;
          const int sh = (int)((((size_t)row * KC + 2 * (g_stage < nstg ? g_stage : 0)) & 3) * 8);
          const uint32_t a0 = (wd >> sh) & 0xFFu, a1 = (wd >> (sh + 8)) & 0xFFu;
          v = a0 | (a0 << 8) | (a1 << 16) | (a1 << 24);
        }
      }
      *reinterpret_cast<uint32_t*>(sfb + (tid & 31) * 16) = v;
    }
    tc::fence_proxy_async_smem();
    __syncthreads();
    const bool first = cc.l == 0;
    const bool last = cc.l == p.spt - 1 || j + 1 == nstages;
    if (tid == 0) {
      tc::fence_after();
      const uint32_t t_sfa = tmem + 16 + 8 * b, t_sfb = t_sfa + 4;
      tc::cp_sf_32x128b_warpx4(t_sfa, tc::smem_desc(tc::smem_addr(sfa), 0, 128));
      tc::cp_sf_32x128b_warpx4(t_sfb, tc::smem_desc(tc::smem_addr(sfb), 0, 128));
      const uint8_t* B = rs + kCodes + kSfRaw;
      if (g_stage < nstg) {
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
          const uint64_t da = tc::smem_desc(tc::smem_addr(A + kk * 256), 128, 1024);
          const uint64_t db = tc::smem_desc(tc::smem_addr(B + kk * 256), 128, 1024);
          tc::mma_mxf8(tmem, da, db, tc::idesc_mxf8(128, NT, kk, kk), (!first || kk > 0) ? 1u : 0u, t_sfa, t_sfb);
        }
      }
      tc::commit(&mma_done[b]);
    }
    uses[b]++;
    if (last) {   // epilogue of the task: accumulator -> out slice
      const bool w = tc::mbar_wait(&mma_done[b], (uses[b] - 1) & 1);
      if (!__syncthreads_and(w)) { ok = false; break; }
      tc::fence_after();
      const int slot = cc.slot;
      const int row = warp * 32 + lane, grow = cc.rt * 128 + row;
      float* outs = p.out + (size_t)cc.sl * p.part_stride;
      const bool any = cc.sl * p.spt < nstg;     // a slice past K's end holds no stage: zeros
      if (slot < 0 && cc.rt == 0 && cc.sl == 0 && tid == 0 && p.miss_count) atomicAdd(p.miss_count, 1);
#pragma unroll
      for (int c = 0; c < NT; c += 8) {
        uint32_t r[8];
        tc::tmem_ld8(tmem + ((uint32_t)(warp * 32) << 16) + c, r);
        tc::tmem_wait_ld();
        if (grow < p.N) {
#pragma unroll
          for (int q = 0; q < 8; q++) {
            const int n = c + q;
            if (n >= pr.z) break;
            const float v = (slot >= 0 && any) ? __uint_as_float(r[q]) : 0.f;
            outs[(size_t)(pr.y + n) * p.out_stride + grow] = v;
          }
        }
      }
      tc::fence_before();
    }
    if (j + 1 < nstages) cur_next(cc, true);
  }
  tcd::cp_wait<0>();
  if (!ok) {   // a wait gave up: record it, let the MMAs issued so far finish, then free TMEM
    if (tid == 0) {
      set_status(p.status, kTimeout);
      tc::commit(&drain);
      tc::mbar_wait(&drain, 0);
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 64);
}

}  // namespace moet

using namespace moet;

// out: [ksplit, rows, N] f32 K-slice partials; K % 128 == 0, N % 16 == 0; rows_per_pair 8 or 16.
void moe_w2_tcd(torch::Tensor a, torch::Tensor sa, c10::optional<torch::Tensor> gather, torch::Tensor pairs,
                torch::Tensor n_pairs, torch::Tensor pool, int64_t codes_off, int64_t scale_off,
                torch::Tensor slot_table, torch::Tensor out, int64_t N, int64_t K, int64_t rows_per_pair,
                c10::optional<torch::Tensor> miss_count, torch::Tensor status) {
  TORCH_CHECK(K % 128 == 0 && N % 16 == 0, "moe_w2_tcd: K % 128, N % 16");
  TORCH_CHECK(a.stride(1) == 1 && a.size(1) == K && a.stride(0) % 16 == 0 &&
              reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0, "moe_w2_tcd: A [rows, K], 16-byte rows");
  TORCH_CHECK(sa.is_contiguous() && sa.size(1) == K / 64 && reinterpret_cast<uintptr_t>(sa.data_ptr()) % 4 == 0,
              "moe_w2_tcd: sA [rows, K/64]");
  TORCH_CHECK(out.dim() == 3 && out.scalar_type() == at::kFloat && out.stride(2) == 1 && out.size(2) == N,
              "moe_w2_tcd: out [ksplit, rows, N] f32");
  TORCH_CHECK(pool.dim() == 2 && codes_off % 16 == 0 && scale_off % 16 == 0 && pool.stride(0) % 16 == 0 &&
              reinterpret_cast<uintptr_t>(pool.data_ptr()) % 16 == 0, "moe_w2_tcd: pool alignment");
  const int nstg = K / 128, ks = out.size(0);
  TORCH_CHECK(ks >= 1 && ks <= nstg, "moe_w2_tcd: 1 <= ksplit <= K / 128");
  TcdArgs p;
  p.A = (const uint8_t*)a.data_ptr(); p.sA = (const uint8_t*)sa.data_ptr(); p.a_stride = a.stride(0);
  p.gather = gather.has_value() && gather->defined() ? gather->data_ptr<int>() : nullptr;
  p.pairs = (const int4*)pairs.data_ptr<int>(); p.n_pairs = n_pairs.data_ptr<int>();
  p.pool = (const uint8_t*)pool.data_ptr(); p.slot_bytes = pool.stride(0);
  p.codes_off = codes_off; p.scale_off = scale_off;
  p.slot_table = slot_table.data_ptr<int>();
  p.out = out.data_ptr<float>(); p.out_stride = out.stride(1); p.part_stride = out.stride(0);
  p.N = N; p.K = K; p.ksplit = ks; p.spt = (nstg + ks - 1) / ks;
  p.miss_count = miss_count.has_value() && miss_count->defined() ? miss_count->data_ptr<int>() : nullptr;
  p.status = status.data_ptr<int>();
  static int n_sm = 0, smem_sm = 0;
  if (!n_sm) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  auto launch = [&](auto kern, size_t smem) {
    moet_allow_max_smem(kern);
    cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    // CTAs per SM from shared memory (1 KB per CTA reserved by the system); registers allow 5,
    // TMEM (64 columns each) 8
    const int per_sm = std::max(1, std::min(4, smem_sm / (int)(smem + 1024 + 64)));
    launch_k(kern, per_sm * n_sm, tcd::kThreads, smem, stream, p);
  };
  static const int na = [] {
    const char* e = getenv("MOET_TCD_NA");
    return e ? atoi(e) : 2;
  }();
  if (rows_per_pair == 8 && na == 3) launch(moe_w2_tcd_kernel<8, 3>, tcd::Cfg<8, 3>::SMEM);
  else if (rows_per_pair == 8) launch(moe_w2_tcd_kernel<8, 2>, tcd::Cfg<8, 2>::SMEM);
  else if (rows_per_pair == 16 && na == 3) launch(moe_w2_tcd_kernel<16, 3>, tcd::Cfg<16, 3>::SMEM);
  else if (rows_per_pair == 16) launch(moe_w2_tcd_kernel<16, 2>, tcd::Cfg<16, 2>::SMEM);
  else TORCH_CHECK(false, "moe_w2_tcd: rows_per_pair must be 8 or 16");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
