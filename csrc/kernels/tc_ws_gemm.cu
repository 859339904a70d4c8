// Warp-specialized, persistent tcgen05 block-scaled "swap-AB" GEMM:
//   out[tok, row] = sum_k act[tok, k] * W[row, k]
// with the weight rows as the M = 128 operand and NT (8..128) tokens as N.
//
// ASRC = 0: W is a 2-bit codebook expert held in a slot pool (fragment-major
//           code plane + UE8M0 block-32 scale plane per slot); work items are
//           (expert pair, 128-row tile).  Pairs come from the padded pair list,
//           so each pair's token rows are NT-aligned and contiguous.
// ASRC = 1: W is dense e4m3 [N, K] with UE8M0 128x128 block scales; work items
//           are (128-token tile, 128-row tile).
// Activations are e4m3 [rows, K] with UE8M0 per-64 scales [rows, K/64]
// (contiguous); for ASRC 0 in the w2 layout, whose in-k32 byte order equals
// the order the decode writes A in, so A and B agree on the physical k order.
//
// One CTA per SM loops over work tiles.  Roles (10 warps):
//   warp 0     producer: per 128-K stage one 4D TMA each for the code chunks
//              and the raw scale bytes of the 8 row blocks (the slot index is a
//              tensor coordinate), or one 4D TMA of dense weights in the UMMA
//              canonical K-major layout; one 4D TMA of the token rows; per tile
//              one bulk copy of the tokens' scale rows.
//   warps 2..9 converters: decode 2-bit codes into the e4m3 A tile (warp =
//              16-row block), build the scale-factor atoms; then epilogue.
//   warp 1     MMA: scale factors into TMEM, 4 block-scaled MMAs per stage,
//              commits stage buffers back to the producer.
// Rings: full/conv/empty per stage, tfull/tempty per tile (scale rows),
// accfull/accempty for the two TMEM accumulators.  Every wait is bounded.
#include <cuda.h>
#include "tcgen05.cuh"
#include "torch_glue.h"

namespace moet {
namespace ws {

MOET_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_addr(bar)) : "memory");
}
MOET_DEVICE void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc::smem_addr(bar)), "r"(bytes) : "memory");
}
MOET_DEVICE void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(tc::smem_addr(dst)), "l"(src), "r"(bytes), "r"(tc::smem_addr(bar)) : "memory");
}
MOET_DEVICE void tma_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
      ::"r"(tc::smem_addr(dst)), "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(tc::smem_addr(bar)) : "memory");
}
MOET_DEVICE void named_sync(int id, int nthreads) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory"); }

MOET_DEVICE bool wait(uint64_t* bar, uint32_t parity, volatile int* err, long long& acc) {
  const long long t0 = clock64();
  const bool ok = tc::mbar_wait(bar, parity);
  acc += clock64() - t0;
  if (!ok) *err = 1;
  return ok;
}

}  // namespace ws

struct WsArgs {
  const uint8_t* act_s; int act_groups;           // [rows, K/64] contiguous
  const int4* pairs; const int* n_pairs;
  const int* slot_table;
  const uint8_t* sW; int sw_cols;
  int T;
  void* out; long long out_stride; int out_f32; const __nv_bfloat16* resid;
  int N, K;
  int* miss_count; int* status;
  long long* dbg_clk;   // per-role cycle counters of CTA 0 (profiling; null in production)
  int dbg;              // measurement switches (0 in production)
};

template <int NT, int ASRC>
struct WsCfg {
  static constexpr int S = NT <= 16 ? 8 : 4;
  static constexpr int A = 16384;
  static constexpr int B = NT * 128 < 1024 ? 1024 : NT * 128;
  static constexpr int CODES = ASRC == 0 ? 4096 : 0;
  static constexpr int SFRAW = ASRC == 0 ? 1024 : 0;   // 8 row blocks x 4 k-blocks x 16 rows (512 B used)
  static constexpr int SF = 512;
  static constexpr int STAGE = A + B + CODES + SFRAW + 2 * SF;
  static constexpr int TCOLS_NEED = 2 * NT + 8 * S;
  static constexpr int TCOLS = TCOLS_NEED <= 32 ? 32 : TCOLS_NEED <= 64 ? 64 : TCOLS_NEED <= 128 ? 128 :
                               TCOLS_NEED <= 256 ? 256 : 512;
};

constexpr int kConvWarps = 16;
constexpr int kConvThreads = kConvWarps * 32;

template <int NT, int ASRC>
__global__ void __launch_bounds__(64 + kConvThreads, 1) tc_ws_kernel(const __grid_constant__ CUtensorMap map_w,
                                                       const __grid_constant__ CUtensorMap map_s,
                                                       const __grid_constant__ CUtensorMap map_b, WsArgs p) {
  using Cf = WsCfg<NT, ASRC>;
  constexpr int S = Cf::S;
  extern __shared__ uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  const int G = p.act_groups;                              // scale bytes per token row
  uint8_t* tsc = sm + S * Cf::STAGE;                        // [2][NT][G] token scale rows (per tile)
  uint8_t* tsw = tsc + 2 * NT * G;                          // [K/128] dense weight scales of the tile row block
  __shared__ uint64_t full[S], conv[S], empty[S], accfull[2], accempty[2], tfull[2], tempty[2], drain;
  __shared__ uint32_t taddr_s;
  __shared__ volatile int err_s;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = p.K, nstages = K / 128;
  const int n_row_tiles = (p.N + 127) / 128;
  const int nwork = ASRC == 0 ? *p.n_pairs : (p.T + NT - 1) / NT;
  const int ntiles = n_row_tiles * nwork;

  if (tid == 0) {
    for (int i = 0; i < S; i++) { tc::mbar_init(&full[i], 1); tc::mbar_init(&conv[i], kConvWarps); tc::mbar_init(&empty[i], 1); }
    for (int i = 0; i < 2; i++) {
      tc::mbar_init(&accfull[i], 1); tc::mbar_init(&accempty[i], kConvWarps);
      tc::mbar_init(&tfull[i], 1); tc::mbar_init(&tempty[i], kConvWarps);
    }
    tc::mbar_init(&drain, 1);
    err_s = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tc::tmem_alloc(&taddr_s, Cf::TCOLS);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = taddr_s;
  volatile int* err = &err_s;

  // tile -> (row tile m0, first token row r0, rows, slot); false for a missing expert
  auto tile_info = [&](int tile, int& m0, int& r0, int& nrows, int& slot) -> bool {
    m0 = (tile % n_row_tiles) * 128;
    const int wi = tile / n_row_tiles;
    if constexpr (ASRC == 0) {
      const int4 pr = p.pairs[wi];
      r0 = pr.y; nrows = pr.z;
      slot = p.slot_table[pr.x];
      return slot >= 0;
    } else {
      r0 = wi * NT; nrows = min(NT, p.T - r0); slot = 0;
      return true;
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer (lane 0)
    if (lane == 0) {
      int st = 0; uint32_t ph = 0; int tb = 0; uint32_t tph = 0;
      uint32_t issued = 0, tissued = 0;           // bit i: slot i has a fill in flight or landed, parity in *_ph
      uint32_t issued_ph = 0, tissued_ph = 0;
      long long t0 = clock64(), tw = 0;
      for (int tile = blockIdx.x; tile < ntiles && !*err; tile += gridDim.x) {
        int m0, r0, nrows, slot;
        if (!tile_info(tile, m0, r0, nrows, slot)) continue;
        if (!ws::wait(&tempty[tb], tph ^ 1, err, tw)) break;
        tissued |= 1u << tb; tissued_ph = (tissued_ph & ~(1u << tb)) | (tph << tb);
        ws::mbar_expect_tx(&tfull[tb], NT * G);
        ws::bulk_g2s(tsc + tb * NT * G, p.act_s + (size_t)r0 * G, NT * G, &tfull[tb]);
        if (++tb == 2) { tb = 0; tph ^= 1; }
        for (int s = 0; s < nstages; s++) {
          if (!ws::wait(&empty[st], ph ^ 1, err, tw)) break;
          uint8_t* stage = sm + st * Cf::STAGE;
          uint8_t* sA = stage; uint8_t* sB = sA + Cf::A; uint8_t* sC = sB + Cf::B; uint8_t* sR = sC + Cf::CODES;
          ws::mbar_expect_tx(&full[st], (ASRC == 0 ? 4096 + 512 : 16384) + NT * 128);
          if constexpr (ASRC == 0) {
            ws::tma_4d(sC, &map_w, 0, 2 * s, m0 / 16, slot, &full[st]);   // 8 row blocks x 2 chunks x 256 B
            ws::tma_4d(sR, &map_s, 0, 4 * s, m0 / 16, slot, &full[st]);   // 8 row blocks x 4 k-blocks x 16 B
          } else {
            ws::tma_4d(sA, &map_w, 0, 0, s * 8, m0 / 8, &full[st]);
          }
          ws::tma_4d(sB, &map_b, 0, 0, s * 8, r0 / 8, &full[st]);
          issued |= 1u << st; issued_ph = (issued_ph & ~(1u << st)) | (ph << st);
          if (++st == S) { st = 0; ph ^= 1; }
        }
      }
      if (*err) {   // a wait gave up: let every copy this thread started land before the CTA exits
        for (int i = 0; i < S; i++)
          if (issued >> i & 1) tc::mbar_wait(&full[i], issued_ph >> i & 1);
        for (int i = 0; i < 2; i++)
          if (tissued >> i & 1) tc::mbar_wait(&tfull[i], tissued_ph >> i & 1);
      }
      if (p.dbg_clk && blockIdx.x == 0) { p.dbg_clk[0] = clock64() - t0; p.dbg_clk[1] = tw; }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (lane 0)
    if (lane == 0) {
      int st = 0; uint32_t ph = 0; int acc = 0; uint32_t aph = 0;
      long long t0 = clock64(), tw = 0, twa = 0;
      for (int tile = blockIdx.x; tile < ntiles && !*err; tile += gridDim.x) {
        int m0, r0, nrows, slot;
        if (!tile_info(tile, m0, r0, nrows, slot)) continue;
        if (!ws::wait(&accempty[acc], aph ^ 1, err, twa)) break;
        tc::fence_after();
        const uint32_t t_acc = tmem + acc * NT;
        for (int s = 0; s < nstages; s++) {
          if (!ws::wait(&conv[st], ph, err, tw)) break;
          tc::fence_after();
          uint8_t* stage = sm + st * Cf::STAGE;
          uint8_t* sA = stage; uint8_t* sB = sA + Cf::A;
          uint8_t* sSFA = sB + Cf::B + Cf::CODES + Cf::SFRAW; uint8_t* sSFB = sSFA + Cf::SF;
          const uint32_t t_sfa = tmem + 2 * NT + 8 * st, t_sfb = t_sfa + 4;
          if (!(p.dbg & 16)) {
            tc::cp_sf_32x128b_warpx4(t_sfa, tc::smem_desc(tc::smem_addr(sSFA), 0, 128));
            tc::cp_sf_32x128b_warpx4(t_sfb, tc::smem_desc(tc::smem_addr(sSFB), 0, 128));
          }
#pragma unroll
          for (int kk = 0; kk < 4 && !(p.dbg & 32); kk++) {
            const uint64_t da = tc::smem_desc(tc::smem_addr(sA + kk * 256), 128, 1024);
            const uint64_t db = tc::smem_desc(tc::smem_addr(sB + kk * 256), 128, 1024);
            tc::mma_mxf8(t_acc, da, db, tc::idesc_mxf8(128, NT, kk, kk), (s > 0 || kk > 0) ? 1u : 0u, t_sfa, t_sfb);
          }
          tc::commit(&empty[st]);
          if (++st == S) { st = 0; ph ^= 1; }
        }
        tc::commit(&accfull[acc]);
        if (++acc == 2) { acc = 0; aph ^= 1; }
      }
      if (*err) {   // a wait gave up: a commit tracks every MMA issued so far; wait for them before TMEM is freed
        tc::commit(&drain);
        tc::mbar_wait(&drain, 0);
      }
      if (p.dbg_clk && blockIdx.x == 0) { p.dbg_clk[2] = clock64() - t0; p.dbg_clk[3] = tw; p.dbg_clk[4] = twa; }
    }
  } else {
    // ------------------------------------------------------------ converters + epilogue (warps 2..9)
    const int ct = tid - 64;                         // 0..kConvThreads-1
    const int cw = ct >> 5;                          // converter warp: (16-row block, 64-K half) unit
    const int g = lane >> 2, t = lane & 3;
    const int quarter = warp & 3;                    // TMEM lane quarter this warp may access
    int st = 0; uint32_t ph = 0; int acc = 0; uint32_t aph = 0; int tb = 0; uint32_t tph = 0;
    long long t0 = clock64(), tw = 0, twa = 0, tepi = 0;
    for (int tile = blockIdx.x; tile < ntiles && !*err; tile += gridDim.x) {
      int m0, r0, nrows, slot;
      if (!tile_info(tile, m0, r0, nrows, slot)) {
        if constexpr (ASRC == 0) {   // missing expert: its output rows are zero
          if ((tile % n_row_tiles) == 0 && ct == 0 && p.miss_count) atomicAdd(p.miss_count, 1);
          for (int i = ct; i < nrows * 128; i += kConvThreads) {
            const int n = i >> 7, row = m0 + (i & 127);
            if (row < p.N) reinterpret_cast<float*>(p.out)[(size_t)(r0 + n) * p.out_stride + row] = 0.f;
          }
        }
        continue;
      }
      if constexpr (ASRC == 1) {
        for (int j = ct; j < nstages; j += kConvThreads) tsw[j] = __ldg(p.sW + (size_t)(m0 >> 7) * p.sw_cols + j);
        ws::named_sync(1, kConvThreads);
      }
      if (!ws::wait(&tfull[tb], tph, err, tw)) break;
      const uint8_t* ts = tsc + tb * NT * G;
      for (int s = 0; s < nstages; s++) {
        if (!ws::wait(&full[st], ph, err, tw)) break;
        uint8_t* stage = sm + st * Cf::STAGE;
        uint8_t* sA = stage; uint8_t* sB = sA + Cf::A; uint8_t* sC = sB + Cf::B; uint8_t* sR = sC + Cf::CODES;
        uint8_t* sSFA = sR + Cf::SFRAW; uint8_t* sSFB = sSFA + Cf::SF;
        if constexpr (ASRC == 0) {
          constexpr uint32_t LUT = 0x4838B8C8u;
          {
            const int rblk = cw >> 1, kl = cw & 1;       // 16 units per stage: 8 row blocks x 2 chunks
            const uint2 w = *reinterpret_cast<const uint2*>(sC + rblk * 512 + kl * 256 + lane * 8);
            const uint32_t lo = w.x, hi = w.y;
            const uint2 ra = make_uint2(prmt(LUT, LUT, lo & 0x3333u), prmt(LUT, LUT, (lo >> 2) & 0x3333u));
            const uint2 rb = make_uint2(prmt(LUT, LUT, (lo >> 16) & 0x3333u), prmt(LUT, LUT, (lo >> 18) & 0x3333u));
            const uint2 ha = make_uint2(prmt(LUT, LUT, hi & 0x3333u), prmt(LUT, LUT, (hi >> 2) & 0x3333u));
            const uint2 hb = make_uint2(prmt(LUT, LUT, (hi >> 16) & 0x3333u), prmt(LUT, LUT, (hi >> 18) & 0x3333u));
            const int row0 = rblk * 16 + g, row1 = row0 + 8, kloc = kl * 64;
            *reinterpret_cast<uint2*>(sA + tc::kmajor_off(row0, kloc + 8 * t, 128)) = ra;
            *reinterpret_cast<uint2*>(sA + tc::kmajor_off(row0, kloc + 32 + 8 * t, 128)) = rb;
            *reinterpret_cast<uint2*>(sA + tc::kmajor_off(row1, kloc + 8 * t, 128)) = ha;
            *reinterpret_cast<uint2*>(sA + tc::kmajor_off(row1, kloc + 32 + 8 * t, 128)) = hb;
          }
          if (ct < 128) {   // raw scale bytes [row block][k-block][16 rows] -> atom, thread = row
            const int m = ct;
            const uint8_t* sp = sR + (m >> 4) * 64 + (m & 15);
            const uint32_t v = (uint32_t)sp[0] | ((uint32_t)sp[16] << 8) | ((uint32_t)sp[32] << 16) | ((uint32_t)sp[48] << 24);
            *reinterpret_cast<uint32_t*>(sSFA + (m & 31) * 16 + (m >> 5) * 4) = v;
          }
        } else {
          if (ct < 128) *reinterpret_cast<uint32_t*>(sSFA + (ct & 31) * 16 + (ct >> 5) * 4) = (uint32_t)tsw[s] * 0x01010101u;
        }
        if (ct < NT) {
          uint32_t v = 0;
          if (ct < nrows) {
            const uint32_t a0 = ts[ct * G + 2 * s], a1 = ts[ct * G + 2 * s + 1];
            v = a0 | (a0 << 8) | (a1 << 16) | (a1 << 24);
          }
          *reinterpret_cast<uint32_t*>(sSFB + (ct & 31) * 16 + (ct >> 5) * 4) = v;
        }
        // each lane makes its own smem writes visible to the async proxy; after the
        // warp converges one lane arrives for the whole warp
        if (!(p.dbg & 8)) tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) ws::mbar_arrive(&conv[st]);
        if (++st == S) { st = 0; ph ^= 1; }
      }
      if (*err) break;
      __syncwarp();
      if (lane == 0) ws::mbar_arrive(&tempty[tb]);
      if (++tb == 2) { tb = 0; tph ^= 1; }
      // ---- epilogue ----
      if (!ws::wait(&accfull[acc], aph, err, twa)) break;
      const long long te = clock64();
      tc::fence_after();
      const int row = quarter * 32 + lane, grow = m0 + row;
      const uint32_t t_acc = tmem + acc * NT + ((uint32_t)(quarter * 32) << 16);
      const int part = cw >> 2;                      // the four warps of a lane quarter split the column chunks
#pragma unroll 1
      for (int c0 = 8 * part; c0 < NT; c0 += 32) {
        uint32_t r[8];
        tc::tmem_ld8(t_acc + c0, r);
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
      tc::fence_before();
      __syncwarp();
      if (lane == 0) ws::mbar_arrive(&accempty[acc]);
      tepi += clock64() - te;
      if (++acc == 2) { acc = 0; aph ^= 1; }
    }
    if (p.dbg_clk && blockIdx.x == 0 && ct == 0) {
      p.dbg_clk[5] = clock64() - t0; p.dbg_clk[6] = tw; p.dbg_clk[7] = twa; p.dbg_clk[8] = tepi;
    }
  }
  tc::fence_before();
  __syncthreads();
  if (tid == 0 && *err) set_status(p.status, kTimeout);
  if (warp == 1) { tc::tmem_dealloc(tmem, Cf::TCOLS); tc::tmem_relinquish(); }
}

// ---------------------------------------------------------------- host side
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                              const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeFn encoder() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    TORCH_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess && f,
                "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeFn>(f);
  }
  return fn;
}
static void encode4d(CUtensorMap* map, const void* base, const cuuint64_t (&dims)[4], const cuuint64_t (&strides)[3],
                     const cuuint32_t (&box)[4], const char* what) {
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = encoder()(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "tensor map encode failed for ", what, " (", (int)r, ")");
}
// Row-major [rows, K] bytes -> boxes in the UMMA canonical K-major no-swizzle layout:
// dims (16 B, 8 rows, K/16 slices, rows/8 groups); box (16, 8, 8, box_rows/8) = one 128-K stage.
static void canonical_map(CUtensorMap* m, const void* base, long long rows, long long K, long long row_stride,
                          int box_rows, const char* what) {
  const cuuint64_t dims[4] = {16, 8, (cuuint64_t)(K / 16), (cuuint64_t)(rows / 8)};
  const cuuint64_t strides[3] = {(cuuint64_t)row_stride, 16, (cuuint64_t)(8 * row_stride)};
  const cuuint32_t box[4] = {16, 8, 8, (cuuint32_t)(box_rows / 8)};
  encode4d(m, base, dims, strides, box, what);
}

template <int NT, int ASRC>
static void launch_ws(const WsArgs& a, const CUtensorMap& mw, const CUtensorMap& ms, const CUtensorMap& mb,
                      cudaStream_t stream) {
  using Cf = WsCfg<NT, ASRC>;
  static int sms = 0;
  if (!sms) { int dev; cudaGetDevice(&dev); cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev); }
  const int smem = Cf::S * Cf::STAGE + 2 * NT * a.act_groups + 256 + 1024;
  TORCH_CHECK(smem <= 227 * 1024, "tc_ws: shared memory budget exceeded (", smem, " bytes)");
  moet_allow_max_smem(tc_ws_kernel<NT, ASRC>);
  tc_ws_kernel<NT, ASRC><<<sms, 64 + kConvThreads, smem, stream>>>(mw, ms, mb, a);
}

}  // namespace moet

using namespace moet;

// Experts over the padded pair list: a [Rp, K] (w2 layout) and sa [Rp, K/64] hold the
// expert-sorted, NT-aligned token rows (Rp a multiple of 8); out [Rp, N] f32.
void ws_moe_w2(torch::Tensor a, torch::Tensor sa, torch::Tensor pairs, torch::Tensor n_pairs, torch::Tensor pool,
               int64_t codes_off, int64_t scale_off, torch::Tensor slot_table, torch::Tensor out, int64_t N,
               int64_t K, int64_t nt, c10::optional<torch::Tensor> miss_count, torch::Tensor status,
               c10::optional<torch::Tensor> dbg_clk) {
  const int dbg_flags = dbg_clk.has_value() && dbg_clk->defined() ? (int)dbg_clk->size(0) - 16 : 0;
  TORCH_CHECK(K % 128 == 0 && N % 128 == 0 && K <= 16384, "ws_moe_w2: K % 128, N % 128, K <= 16384");
  TORCH_CHECK(a.stride(1) == 1 && a.size(1) == K && a.stride(0) % 16 == 0 && a.size(0) % 8 == 0, "ws_moe_w2: activations");
  TORCH_CHECK(sa.is_contiguous() && sa.size(1) == K / 64 && sa.size(0) >= a.size(0), "ws_moe_w2: activation scales");
  TORCH_CHECK((8 * (K / 64)) % 16 == 0, "ws_moe_w2: K/64 scale rows must give 16-byte aligned tiles");
  TORCH_CHECK(out.scalar_type() == at::kFloat && pool.dim() == 2 && pool.stride(0) % 16 == 0, "ws_moe_w2: out / pool");
  WsArgs p{};
  p.act_s = (const uint8_t*)sa.data_ptr(); p.act_groups = K / 64;
  p.pairs = (const int4*)pairs.data_ptr<int>(); p.n_pairs = n_pairs.data_ptr<int>();
  p.slot_table = slot_table.data_ptr<int>();
  p.out = out.data_ptr(); p.out_stride = out.stride(0); p.out_f32 = 1;
  p.N = N; p.K = K;
  p.miss_count = miss_count.has_value() && miss_count->defined() ? miss_count->data_ptr<int>() : nullptr;
  p.status = status.data_ptr<int>();
  p.dbg_clk = dbg_clk.has_value() && dbg_clk->defined() ? (long long*)dbg_clk->data_ptr() : nullptr;
  p.dbg = dbg_flags > 0 ? dbg_flags : 0;
  CUtensorMap mw{}, ms{}, mb{};
  const uint8_t* pool_p = (const uint8_t*)pool.data_ptr();
  const long long slots = pool.size(0), sb = pool.stride(0);
  {
    const cuuint64_t dims[4] = {256, (cuuint64_t)(K / 64), (cuuint64_t)(N / 16), (cuuint64_t)slots};
    const cuuint64_t strides[3] = {256, (cuuint64_t)(K / 64) * 256, (cuuint64_t)sb};
    const cuuint32_t box[4] = {256, 2, 8, 1};
    encode4d(&mw, pool_p + codes_off, dims, strides, box, "code plane");
  }
  {
    const cuuint64_t dims[4] = {16, (cuuint64_t)(K / 32), (cuuint64_t)(N / 16), (cuuint64_t)slots};
    const cuuint64_t strides[3] = {16, (cuuint64_t)(K / 32) * 16, (cuuint64_t)sb};
    const cuuint32_t box[4] = {16, 4, 8, 1};
    encode4d(&ms, pool_p + scale_off, dims, strides, box, "scale plane");
  }
  canonical_map(&mb, a.data_ptr(), a.size(0), K, a.stride(0), (int)nt, "token rows");
  auto stream = at::cuda::getCurrentCUDAStream();
  switch (nt) {
    case 8: launch_ws<8, 0>(p, mw, ms, mb, stream); break;
    case 16: launch_ws<16, 0>(p, mw, ms, mb, stream); break;
    case 128: launch_ws<128, 0>(p, mw, ms, mb, stream); break;
    default: TORCH_CHECK(false, "ws_moe_w2: token tile must be 8, 16 or 128");
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Dense FP8 GEMM out[T, N] (+ resid) = a[T, K] * w[N, K]^T with 128-token tiles.
// a / sa must have at least ceil(T / 128) * 128 rows (padded workspace); sa contiguous [rows, K/64].
void ws_gemm_fp8(torch::Tensor a, torch::Tensor sa, torch::Tensor w, torch::Tensor sw, torch::Tensor out,
                 c10::optional<torch::Tensor> resid, int64_t T, torch::Tensor status) {
  const int K = a.size(1), N = w.size(0);
  const long long Tp = (T + 127) / 128 * 128;
  TORCH_CHECK(K % 128 == 0 && K <= 16384 && w.size(1) == K && w.is_contiguous() && N % 8 == 0,
              "ws_gemm_fp8: K % 128 (<= 16384), N % 8, contiguous W");
  TORCH_CHECK(a.stride(1) == 1 && a.stride(0) % 16 == 0 && a.size(0) >= Tp, "ws_gemm_fp8: activation rows padded to 128");
  TORCH_CHECK(sa.is_contiguous() && sa.size(1) == K / 64 && sa.size(0) >= Tp && (128 * (K / 64)) % 16 == 0,
              "ws_gemm_fp8: activation scales");
  if (T == 0) return;
  WsArgs p{};
  p.act_s = (const uint8_t*)sa.data_ptr(); p.act_groups = K / 64;
  p.sW = (const uint8_t*)sw.data_ptr(); p.sw_cols = sw.size(1);
  p.T = (int)T;
  p.out = out.data_ptr(); p.out_stride = out.stride(0); p.out_f32 = out.scalar_type() == at::kFloat;
  p.resid = resid.has_value() && resid->defined() ? (const __nv_bfloat16*)resid->data_ptr() : nullptr;
  if (p.resid) TORCH_CHECK(resid->stride(0) == out.stride(0), "ws_gemm_fp8: resid layout");
  p.N = N; p.K = K; p.status = status.data_ptr<int>();
  CUtensorMap mw{}, ms{}, mb{};
  canonical_map(&mw, w.data_ptr(), N, K, K, 128, "weights");
  canonical_map(&mb, a.data_ptr(), Tp, K, a.stride(0), 128, "activations");
  launch_ws<128, 1>(p, mw, ms, mb, at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
