// Persistent, warp-specialised grouped FP8 Wgrad GEMM for sm_100a (B200).
//
// Computes, per expert e and output tile (m0, n0):
//   out[e, m, n] = sum_b  sa[b, m] * sb[b, n] * ( sum_{k in b} A[m, k] * B[n, k] )
// with A = lhs FP8 [M][pitch] and B = rhs FP8 [N][pitch] (K contiguous), b the
// expert's 128-row scale blocks. This is the math of the reference kernel
// Fp8ScaledWgradSm90 (src/sm90_fp8_wgrad/gemm_sm90.py:1211-2321): a fresh
// tensor-core partial per 128-row K block (mma_scaled_128k, :3910-4105),
// promoted into an fp32 accumulator with the rank-1 scale product
// (promote_scaled_acc_epilogue_staged, :5023-5085), converted to BF16 in the
// epilogue (:2211-2290).
//
// B200 design (not a translation of the SM90 kernel):
//   warp 0      : TMA producer. A/B tiles (128 x 128 B, BN x 128 B, 128B
//                 swizzle) into a STAGES-deep shared-memory ring; the per-block
//                 scale vectors sa[128], sb[BN] via 1-D bulk copies into a
//                 separate SCALE_STAGES-deep ring.
//   warp 1      : MMA issuer. One elected lane issues 4 x tcgen05.mma
//                 (kind::f8f6f4, 128 x BN x 32) per K block into one of two
//                 TMEM partial buffers, then tcgen05.commit frees the smem
//                 stage and signals the partial as ready.
//   warps 2, 3  : idle (complete warpgroup 0, which gives registers away).
//   warps 4..    : promotion + epilogue (4, 8 or 16 warps, see Cfg). tcgen05.ld
//                 the partial (thread = TMEM lane = output row), final +=
//                 (raw * sb[n]) * sa[m] with packed f32x2 FMA, release the TMEM
//                 buffer so the tensor pipe computes block b+1 while block b is
//                 promoted. At tile end: fp32 -> BF16 (or fp32), swizzled smem
//                 staging, TMA store (with accumulate, the previous output is
//                 first TMA-loaded into the same staging area and added).
// The serialised WGMMA -> wait -> promote chain of the SM90 kernel
// (gemm_sm90.py:3945, 4023) becomes a two-deep TMEM pipeline here.
//
// Tile schedule: static persistent round robin over
//   tile t -> (expert_order[t / tiles_per_expert], m_tile, n_tile)
// with n fastest; expert_order is LPT (most K blocks first) when supplied.
// Experts with no rows still produce their (zero) tiles, as the reference
// does (gemm_sm90.py:3933).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "ptx.cuh"
#include "wgrad_gemm.cuh"

namespace wgrad {

// Per-role cycle counters (build with -DWGRAD_PROFILE=1; read and cleared by
// sm100_wgrad_profile_counters). One lane of the producer, the MMA warp and
// the first promotion warp of every CTA times its waits and work with clock64;
// the CTA's sums go to g_wgrad_prof at exit. Slots: see kProf* in
// wgrad_gemm.cuh. Off by default: the product build has no timing code.
#if WGRAD_PROFILE
__device__ unsigned long long g_wgrad_prof[kProfSlots];
#define WGRAD_PROF_T(v) const long long v = clock64()
#define WGRAD_PROF_ADD(slot, t0) \
  do {                           \
    if (prof_lane) s_prof[slot] += static_cast<unsigned long long>(clock64() - (t0)); \
  } while (0)
#define WGRAD_PROF_INC(slot) \
  do {                       \
    if (prof_lane) s_prof[slot] += 1ull; \
  } while (0)
#else
#define WGRAD_PROF_T(v) ((void)0)
#define WGRAD_PROF_ADD(slot, t0) ((void)0)
#define WGRAD_PROF_INC(slot) ((void)0)
#endif
#if WGRAD_PROFILE
#define WGRAD_PROF_PTR s_prof, s_issue
#define WGRAD_PROF_LATENCY(stage)                                                                   \
  do {                                                                                           \
    if (prof_lane) s_prof[kProfLoadLatency] += static_cast<unsigned long long>(clock64() - s_issue[stage]); \
  } while (0)
#else
#define WGRAD_PROF_PTR nullptr, nullptr
#define WGRAD_PROF_LATENCY(stage) ((void)0)
#endif

// Event trace of CTAs 0 and 1 over their first kTraceBlocks K blocks (build
// with -DWGRAD_TRACE=1; read with sm100_wgrad_trace_read in such builds):
// SM clock64 stamps of the MMA issuer's and the first promotion warp's steps.
#ifndef WGRAD_TRACE
#define WGRAD_TRACE 0
#endif
constexpr int kTraceBlocks = 64, kTraceEvents = 8;
enum TraceEv : int { kTrMmaReady = 0, kTrMmaIssued = 1, kTrEpiWaitStart = 2, kTrEpiReady = 3, kTrEpiReleased = 4,
                     kTrEpiDone = 5, kTrMmaHalfReady = 6, kTrMmaHalfIssued = 7 };
#if WGRAD_TRACE
__device__ unsigned long long g_wgrad_trace[2][kTraceBlocks][kTraceEvents];
#define WGRAD_TRACE_EV(ev, b)                                                                   \
  do {                                                                                          \
    if (blockIdx.x < 2 && (b) < kTraceBlocks && (threadIdx.x & 31) == 0)                        \
      g_wgrad_trace[blockIdx.x][(b)][(ev)] = static_cast<unsigned long long>(clock64());        \
  } while (0)
#else
#define WGRAD_TRACE_EV(ev, b) ((void)0)
#endif

namespace {

constexpr int BM = 128;
constexpr int BK = 128;  // scale block == K block, bytes per row of an FP8 tile
constexpr int SCALE_STAGES = 6;
constexpr int FIRST_EPI_WARP = 4;

// Promotion warps: EPI = 4, 8 or 16 (one, two or four per TMEM lane quarter);
// each owns 32 rows x BN / (EPI / 4) columns. 16 warps keep more TMEM loads,
// scale loads and output stores in flight (better for short-K, HBM-bound
// launches); 8 warps carry fewer per-warp fixed costs (better for long K).
// EPI = 12 (with BN = 192) puts three 64-column warps on each sub-partition.
// EPI = 4 (with BN = 128) runs two CTAs per SM: two independent pipelines on
// different tiles whose promotion warps share each SM sub-partition, so the
// stalls of one fill the FMA pipe with the other's work.
// Register split: the launch gives THREADS x (65536 / (THREADS x CTAs per SM)
// rounded down to 8) registers; warpgroup 0 drops to REGS_CONTROL and the
// promotion warps take the rest: 16 warps: 640 x 96 = 128 x 32 + 512 x 112;
// 8 warps: 384 x 168 >= 128 x 56 + 256 x 224; 4 warps, 2 CTAs: 256 x 128 =
// 128 x 56 + 128 x 200.
#ifndef WGRAD_FRAG16
#define WGRAD_FRAG16 1
#endif

template <int BN, int EPI, bool PAIR = false>
struct Cfg {
  static constexpr int EPI_WARPS = EPI;
  static constexpr int THREADS = 32 * (4 + EPI_WARPS);
  static constexpr int CTAS_PER_SM = EPI_WARPS == 4 ? 2 : 1;
  // A pair CTA holds half of B, so a stage is 32 KB instead of 48 KB.
  static constexpr int STAGES = PAIR ? 4 : (EPI_WARPS == 4 ? 2 : 3);
  static constexpr uint32_t REGS_CONTROL = EPI_WARPS == 16 ? 32 : (EPI_WARPS == 12 ? 40 : 56);
  static constexpr uint32_t REGS_EPILOGUE =
      EPI_WARPS == 16 ? 112 : (EPI_WARPS == 12 ? 152 : (EPI_WARPS == 4 ? 200 : 224));
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // rows of B this CTA loads
  static constexpr int B_BYTES = B_ROWS * BK;
  static constexpr int SCALE_FLOATS = BM + BN;
  static constexpr int SSTAGES = SCALE_STAGES;  // scale-vector ring depth
  static constexpr int COLS_PER_WARP = BN / (EPI_WARPS / 4);  // EPI_WARPS / 4 column groups
  // tcgen05.ld columns per load: 32 when two such buffers fit beside the accumulator
  static constexpr int CHUNK = REGS_EPILOGUE >= COLS_PER_WARP + 80 ? 32 : 16;
  // Promotion in the 16x256b fragment layout (two rows and a column pair per
  // thread): 8-byte column-scale loads shared by 8 lanes' rows instead of a
  // 16-byte broadcast per 4 columns, a quarter of the shared-memory wavefronts.
  static constexpr bool FRAG16 = WGRAD_FRAG16 != 0 && (EPI_WARPS == 8 || EPI_WARPS == 16) && BN == 256;
  static constexpr int GC = CHUNK / 8;  // 8-column groups per chunk of the fragment layout
  static constexpr int CHUNKS = COLS_PER_WARP / CHUNK;
  static constexpr int OUT_STAGE_BYTES_PER_WARP =
      COLS_PER_WARP * 32 * 2 >= 8192 ? 8192 : 4096;
  // double-buffered partial, allocated as a power of two (192-wide tiles use 384 of 512)
  static constexpr int TMEM_COLS = 2 * BN <= 256 ? 256 : 512;
  static constexpr int SMEM_BYTES = STAGES * (A_BYTES + B_BYTES) + EPI_WARPS * OUT_STAGE_BYTES_PER_WARP +
                                    SSTAGES * SCALE_FLOATS * 4 + 512 /*barriers*/ + 1024 /*align*/;
  static_assert(128 * REGS_CONTROL + 32 * EPI_WARPS * REGS_EPILOGUE <=
                    THREADS * ((65536 / (THREADS * CTAS_PER_SM)) & ~7),
                "register split exceeds the launch allocation");
};

template <int N>
__device__ __forceinline__ void tmem_ld_chunk(uint32_t taddr, uint32_t (&r)[N]) {
  if constexpr (N == 32) tmem_ld_32x32b_x32(taddr, r);
  else tmem_ld_32x32b_x16(taddr, r);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// Tile a persistent CTA (or CTA pair) `begin` of `stride` takes in round r.
// CTA pairs walk the (LPT expert, m, n) list alternately forward and
// backward (boustrophedon), so over two rounds every pair gets one tile from
// the costlier and one from the cheaper end of each stretch of the sorted
// list (measured 1-3 % faster for pairs; neutral to slightly slower for the
// single-CTA tiles, which keep the plain round robin).
template <bool SNAKE>
__device__ __forceinline__ int sched_tile(int r, int begin, int stride) {
  return SNAKE ? r * stride + ((r & 1) ? stride - 1 - begin : begin) : r * stride + begin;
}

struct TileCoord {
  int e, m0, n0;
};

// Tile -> (expert, first row of this CTA, first column). p.bm is the tile's M
// (256 for a CTA pair, whose odd CTA starts row_off = 128 rows further).
__device__ __forceinline__ TileCoord decode_tile(const GemmParams& p, int tile, int row_off = 0) {
  const int e_slot = tile / p.tiles_per_expert;
  const int local = tile - e_slot * p.tiles_per_expert;
  const int tm = local / p.tiles_n;
  const int tn = local - tm * p.tiles_n;
  TileCoord c;
  c.e = p.expert_order != nullptr ? __ldg(p.expert_order + e_slot) : e_slot;
  c.m0 = tm * p.bm + row_off;
  c.n0 = tn * p.bn;
  return c;
}

// TMA producer (one thread): for every K block of every tile this CTA owns,
// the A and B operand tiles into the STAGES-deep ring and the block's A / B
// scale vectors into the SCALE_STAGES-deep scale ring. In a CTA pair (PAIR)
// each CTA loads its own 128 rows of A and its half of B's rows, and both
// loads complete on the even CTA's full barrier, whose producer announces the
// bytes of both; at the end each producer waits until the MMA has released
// every stage it filled, so no release arrives after this CTA has exited.
template <class C, int BN, bool PAIR = false>
__device__ __forceinline__ void run_producer(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b, const GemmParams& p,
                                             uint8_t* s_a, uint8_t* s_b, float* s_scale, uint64_t* full_bar,
                                             uint64_t* empty_bar, uint64_t* sfull_bar, uint64_t* sempty_bar,
                                             volatile int* abort_flag, unsigned long long* s_prof,
                                             long long* issue_clock, int tile_begin = -1, int tile_stride = 0,
                                             uint32_t rank = 0) {
  if (tile_begin < 0) {
    tile_begin = blockIdx.x;
    tile_stride = gridDim.x;
  }
#if WGRAD_PROFILE
  const bool prof_lane = true;  // called by the producer lane only
#else
  (void)s_prof;
#endif
  int stage = 0, sstage = 0;
  uint32_t phase = 0, sphase = 0;
  bool ok = true;
  for (int r = 0, tile = tile_begin; r * tile_stride < p.num_tiles && ok; tile = sched_tile<PAIR>(++r, tile_begin, tile_stride)) {
    if (tile >= p.num_tiles) continue;
    const TileCoord tc = decode_tile(p, tile, static_cast<int>(rank) * BM);
    const int kb0 = __ldg(p.block_offsets + tc.e);
    const int nkb = __ldg(p.block_offsets + tc.e + 1) - kb0;
    const int krow0 = __ldg(p.k_row_offsets + tc.e);
    // the odd CTA of a pair may lie wholly below the last row of M
    const uint32_t a_scale_bytes = static_cast<uint32_t>(max(0, min(BM, p.m - tc.m0))) * 4u;
    const uint32_t b_scale_bytes = static_cast<uint32_t>(min(BN, p.n - tc.n0)) * 4u;
    for (int kb = 0; kb < nkb && ok; ++kb) {
      WGRAD_PROF_T(tw0);
      ok = mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, kDevTimeoutProducer);
      WGRAD_PROF_ADD(kProfProducerWaitStage, tw0);
      if (!ok) break;
      if (issue_clock != nullptr) issue_clock[stage] = clock64();  // profile builds only
      // Test-only failure injection: announce the first stage's bytes but
      // issue no copy, so the stage never fills and the bounded waits of
      // the consumers expire (device error word, clean exit).
      const bool withhold = p.inject == kInjectWithholdFirstLoad && r == 0 && kb == 0;
      if constexpr (PAIR) {
        const uint32_t leader_full = cluster_addr(&full_bar[stage], 0);
        if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * (C::A_BYTES + C::B_BYTES));
        if (!withhold) {
          tma_load_2d_pair(s_a + stage * C::A_BYTES, &tmap_a, leader_full, krow0 + kb * BK, tc.m0);
          tma_load_2d_pair(s_b + stage * C::B_BYTES, &tmap_b, leader_full, krow0 + kb * BK,
                           tc.n0 + static_cast<int>(rank) * C::B_ROWS);
        }
      } else {
        mbar_arrive_expect_tx(&full_bar[stage], C::A_BYTES + C::B_BYTES);
        if (!withhold) {
          tma_load_2d(s_a + stage * C::A_BYTES, &tmap_a, &full_bar[stage], krow0 + kb * BK, tc.m0);
          tma_load_2d(s_b + stage * C::B_BYTES, &tmap_b, &full_bar[stage], krow0 + kb * BK, tc.n0);
        }
      }
      if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }

      WGRAD_PROF_T(tw1);
      ok = mbar_wait(&sempty_bar[sstage], sphase ^ 1u, abort_flag, kDevTimeoutProducer);
      WGRAD_PROF_ADD(kProfProducerWaitScales, tw1);
      if (!ok) break;
      float* dst = s_scale + sstage * C::SCALE_FLOATS;
      const size_t blk = static_cast<size_t>(kb0 + kb);
      mbar_arrive_expect_tx(&sfull_bar[sstage], a_scale_bytes + b_scale_bytes);
      if (a_scale_bytes > 0) bulk_load_1d(dst, p.sa + blk * p.m + tc.m0, a_scale_bytes, &sfull_bar[sstage]);
      bulk_load_1d(dst + BM, p.sb + blk * p.n + tc.n0, b_scale_bytes, &sfull_bar[sstage]);
      if (++sstage == C::SSTAGES) { sstage = 0; sphase ^= 1u; }
    }
  }
  if constexpr (PAIR) {
    // Drain: every stage filled so far has been released by the MMA.
    for (int i = 0; i < C::STAGES && ok; ++i) {
      ok = mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, kDevTimeoutProducer);
      if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
    }
  }
}

// Writes one warp's finished 32 rows x COLS columns (fin, fp32) of tile tc:
// BF16 (or fp32) into the warp's swizzled staging area, then TMA stores of
// 32-row boxes clipped to the output; with accumulate the previous output
// boxes are first loaded through the same tensor map and added. fin holds
// groups of GCOLS columns, GSTRIDE output columns apart (contiguous when
// GSTRIDE == GCOLS). BF16 boxes are BOXC columns wide: 64 (128-byte rows,
// 128B swizzle) or 32 (64-byte rows, 64B swizzle; the output tensor map must
// match); fp32 boxes are 32 columns (128B swizzle). The caller has waited for
// the warp's previous store to finish reading the staging area. Returns
// false when a wait gave up.
// accumulate: the previous output boxes come in through the same tensor map
// and swizzled staging layout the store uses (TMA load into this warp's
// staging area, bounded wait), so each thread adds its own elements.
// Box b of the round covers output columns [col_of(b), +box width).
template <class ColOf>
__device__ __forceinline__ bool load_previous_boxes(const CUtensorMap& tmap_out, const GemmParams& p,
                                                    const TileCoord& tc, int quarter, int lane, uint8_t* stage_out,
                                                    uint64_t* oldout_bar, uint32_t& oldout_phase,
                                                    volatile int* abort_flag, int nboxes, int box_bytes,
                                                    ColOf col_of) {
  if (lane == 0) {
    uint32_t bytes = 0;
    for (int b = 0; b < nboxes; ++b) bytes += col_of(b) < p.n ? box_bytes : 0u;
    mbar_arrive_expect_tx(oldout_bar, bytes);
    for (int b = 0; b < nboxes; ++b) {
      const int c = col_of(b);
      if (c < p.n) tma_load_3d(stage_out + b * box_bytes, &tmap_out, oldout_bar, c, tc.m0 + quarter * 32, tc.e);
    }
  }
  const bool landed = mbar_wait(oldout_bar, oldout_phase, abort_flag, kDevTimeoutEpilogue);
  if (!landed) {
    // Giving up (timeout, or another role aborted): let this warp's own
    // load land before the CTA exits. Bounded, regardless of the abort flag.
    const uint32_t addr = smem_u32(oldout_bar);
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(addr, oldout_phase) && globaltimer_ns() - t0 < WGRAD_WAIT_TIMEOUT_NS) {
    }
  }
  oldout_phase ^= 1u;
  return __all_sync(0xffffffffu, landed);
}

template <int COLS, int OUT_STAGE_BYTES, int GSTRIDE = 64, int GCOLS = 64, int BOXC = 64>
__device__ __forceinline__ bool store_warp_tile(float (&fin)[COLS], const CUtensorMap& tmap_out, const GemmParams& p,
                                                const TileCoord& tc, int quarter, int lane, int col0,
                                                uint8_t* stage_out, uint64_t* oldout_bar, uint32_t& oldout_phase,
                                                volatile int* abort_flag) {
  static_assert(BOXC == 64 || BOXC == 32, "bf16 box width");
  static_assert(GCOLS % BOXC == 0 && GCOLS % 32 == 0, "boxes never straddle a column group");
  const uint32_t stage_addr = smem_u32(stage_out);
  bool ok = true;
  const bool rows_in = (tc.m0 + quarter * 32) < p.m;
  const uint32_t swz = static_cast<uint32_t>(lane & 7);
  auto colof = [&](int f) -> int { return col0 + (f / GCOLS) * GSTRIDE + (f % GCOLS); };
  auto load_previous = [&](int nboxes, int box_cols, int box_bytes, int first_box) -> bool {
    return load_previous_boxes(tmap_out, p, tc, quarter, lane, stage_out, oldout_bar, oldout_phase, abort_flag,
                               nboxes, box_bytes, [&](int b) { return colof((first_box + b) * box_cols); });
  };
  if (!p.out_f32) {
    // bf16: boxes of 32 rows x BOXC columns, BOX_BYTES each, PER_ROUND boxes
    // per staging round. Row `lane` of a box holds CH 16-byte chunks, chunk c
    // stored at chunk c ^ (swizzle row bits): 128B swizzle XORs with
    // lane % 8, 64B swizzle with (lane / 2) % 4.
    constexpr int BOX_BYTES = 32 * BOXC * 2;
    constexpr int CH = BOXC / 8;
    constexpr int BOXES = COLS / BOXC;
    constexpr int PER_ROUND = OUT_STAGE_BYTES / BOX_BYTES < BOXES ? OUT_STAGE_BYTES / BOX_BYTES : BOXES;
    const uint32_t rsw = BOXC == 64 ? swz : static_cast<uint32_t>((lane >> 1) & 3);
#pragma unroll
    for (int bx0 = 0; bx0 < BOXES; bx0 += PER_ROUND) {
      if (bx0 > 0) {
        if (lane == 0) bulk_wait_group_read0();
        __syncwarp();
      }
      if (p.accumulate && rows_in) {
        ok = load_previous(PER_ROUND, BOXC, BOX_BYTES, bx0);
        if (!ok) return false;
#pragma unroll
        for (int bi = 0; bi < PER_ROUND; ++bi) {
          const uint32_t box = stage_addr + bi * BOX_BYTES + lane * (BOXC * 2);
#pragma unroll
          for (int ch = 0; ch < CH; ++ch) {
            const uint4 w = ld_shared_v4(box + ((ch ^ rsw) << 4));
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
            float* v = &fin[(bx0 + bi) * BOXC + ch * 8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ww[i]));
              v[2 * i] += f.x;
              v[2 * i + 1] += f.y;
            }
          }
        }
      }
#pragma unroll
      for (int bi = 0; bi < PER_ROUND; ++bi) {
        const uint32_t box = stage_addr + bi * BOX_BYTES + lane * (BOXC * 2);
#pragma unroll
        for (int ch = 0; ch < CH; ++ch) {
          const float* v = &fin[(bx0 + bi) * BOXC + ch * 8];
          st_shared_v4(box + ((ch ^ rsw) << 4), pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                       pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && rows_in) {
#pragma unroll
        for (int bi = 0; bi < PER_ROUND; ++bi) {
          const int c = colof((bx0 + bi) * BOXC);
          if (c < p.n) tma_store_3d(&tmap_out, stage_out + bi * BOX_BYTES, c, tc.m0 + quarter * 32, tc.e);
        }
        bulk_commit_group();
      }
    }
  } else {
    // fp32: boxes of 32 rows x 32 columns, PER_ROUND boxes per staging round.
    constexpr int BOXES = COLS / 32;
    constexpr int PER_ROUND = OUT_STAGE_BYTES / 4096;
#pragma unroll
    for (int bx0 = 0; bx0 < BOXES; bx0 += PER_ROUND) {
      if (bx0 > 0) {
        if (lane == 0) bulk_wait_group_read0();
        __syncwarp();
      }
      if (p.accumulate && rows_in) {
        ok = load_previous(PER_ROUND, 32, 4096, bx0);
        if (!ok) return false;
#pragma unroll
        for (int bi = 0; bi < PER_ROUND; ++bi) {
          const uint32_t box = stage_addr + bi * 4096 + lane * 128;
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            const uint4 w = ld_shared_v4(box + ((ch ^ swz) << 4));
            float* v = &fin[(bx0 + bi) * 32 + ch * 4];
            v[0] += __uint_as_float(w.x);
            v[1] += __uint_as_float(w.y);
            v[2] += __uint_as_float(w.z);
            v[3] += __uint_as_float(w.w);
          }
        }
      }
#pragma unroll
      for (int bi = 0; bi < PER_ROUND; ++bi) {
        const uint32_t box = stage_addr + bi * 4096 + lane * 128;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const float* v = &fin[(bx0 + bi) * 32 + ch * 4];
          st_shared_v4(box + ((ch ^ swz) << 4), __float_as_uint(v[0]), __float_as_uint(v[1]),
                       __float_as_uint(v[2]), __float_as_uint(v[3]));
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && rows_in) {
#pragma unroll
        for (int bi = 0; bi < PER_ROUND; ++bi) {
          const int c = colof((bx0 + bi) * 32);
          if (c < p.n) tma_store_3d(&tmap_out, stage_out + bi * 4096, c, tc.m0 + quarter * 32, tc.e);
        }
        bulk_commit_group();
      }
    }
  }
  return ok;
}

// Accumulator element f of a promotion warp in the 16x256b fragment layout
// (see tmem_ld_16x256b_x4): chunks of GC 8-column groups, each chunk holding
// the warp's upper 16 rows then its lower 16, four registers per group.
// Row within the warp's 32 rows and column within its COLS columns.
template <int GC>
__device__ __forceinline__ int frag_row(int f, int lane) {
  return 16 * ((f % (8 * GC)) / (4 * GC)) + 8 * ((f % 4) >> 1) + (lane >> 2);
}
template <int GC>
__device__ __forceinline__ int frag_col(int f, int lane) {
  return 8 * ((f / (8 * GC)) * GC + (f % (4 * GC)) / 4) + 2 * (lane & 3) + (f & 1);
}

__device__ __forceinline__ uint32_t ld_shared_b32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_shared_b32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint2 ld_shared_v2(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_shared_v2(uint32_t addr, uint32_t a, uint32_t b) {
  asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(addr), "r"(a), "r"(b) : "memory");
}

// store_warp_tile for an accumulator in the fragment layout: the same boxes,
// staging swizzle and TMA stores, each thread writing its column pairs
// (4 bytes of bf16 or 8 bytes of fp32) into the rows it holds. Within one
// store instruction the warp covers 8 consecutive rows at 8 different
// swizzled 16-byte positions, so the 32 lanes hit 32 different banks.
template <int COLS, int OUT_STAGE_BYTES, int GC>
__device__ __forceinline__ bool store_warp_tile_frag(float (&fin)[COLS], const CUtensorMap& tmap_out,
                                                     const GemmParams& p, const TileCoord& tc, int quarter, int lane,
                                                     int col0, uint8_t* stage_out, uint64_t* oldout_bar,
                                                     uint32_t& oldout_phase, volatile int* abort_flag) {
  const uint32_t stage_addr = smem_u32(stage_out);
  const bool rows_in = (tc.m0 + quarter * 32) < p.m;
  const uint32_t rsw = static_cast<uint32_t>((lane >> 2) & 7);  // every row this thread holds is == lane / 4 mod 8
  constexpr int BOXC = 64;  // bf16 box: 32 rows x 64 columns, 128-byte rows (128B swizzle)
  if (!p.out_f32) {
    constexpr int BOX_BYTES = 32 * BOXC * 2;
    constexpr int BOXES = COLS / BOXC;
    constexpr int PER_ROUND = OUT_STAGE_BYTES / BOX_BYTES < BOXES ? OUT_STAGE_BYTES / BOX_BYTES : BOXES;
#pragma unroll
    for (int bx0 = 0; bx0 < BOXES; bx0 += PER_ROUND) {
      if (bx0 > 0) {
        if (lane == 0) bulk_wait_group_read0();
        __syncwarp();
      }
      auto addr_of = [&](int f) -> uint32_t {
        const int c = frag_col<GC>(f, lane);
        const int r = frag_row<GC>(f, lane);
        return stage_addr + (c / BOXC - bx0) * BOX_BYTES + r * (BOXC * 2) +
               ((static_cast<uint32_t>((c % BOXC) >> 3) ^ rsw) << 4) + 2 * (c & 7);
      };
      if (p.accumulate && rows_in) {
        if (!load_previous_boxes(tmap_out, p, tc, quarter, lane, stage_out, oldout_bar, oldout_phase, abort_flag,
                                 PER_ROUND, BOX_BYTES, [&](int b) { return col0 + (bx0 + b) * BOXC; }))
          return false;
#pragma unroll
        for (int f = 0; f < COLS; f += 2) {
          if (frag_col<GC>(f, 0) / BOXC < bx0 || frag_col<GC>(f, 0) / BOXC >= bx0 + PER_ROUND) continue;
          const uint32_t w = ld_shared_b32(addr_of(f));
          const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
          fin[f] += v.x;
          fin[f + 1] += v.y;
        }
      }
#pragma unroll
      for (int f = 0; f < COLS; f += 2) {
        if (frag_col<GC>(f, 0) / BOXC < bx0 || frag_col<GC>(f, 0) / BOXC >= bx0 + PER_ROUND) continue;
        st_shared_b32(addr_of(f), pack_bf16x2(fin[f], fin[f + 1]));
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && rows_in) {
#pragma unroll
        for (int bi = 0; bi < PER_ROUND; ++bi) {
          const int c = col0 + (bx0 + bi) * BOXC;
          if (c < p.n) tma_store_3d(&tmap_out, stage_out + bi * BOX_BYTES, c, tc.m0 + quarter * 32, tc.e);
        }
        bulk_commit_group();
      }
    }
  } else {
    // fp32: boxes of 32 rows x 32 columns (128-byte rows), PER_ROUND boxes per round.
    constexpr int BOXES = COLS / 32;
    constexpr int PER_ROUND = OUT_STAGE_BYTES / 4096;
#pragma unroll
    for (int bx0 = 0; bx0 < BOXES; bx0 += PER_ROUND) {
      if (bx0 > 0) {
        if (lane == 0) bulk_wait_group_read0();
        __syncwarp();
      }
      auto addr_of = [&](int f) -> uint32_t {
        const int c = frag_col<GC>(f, lane);
        const int r = frag_row<GC>(f, lane);
        return stage_addr + (c / 32 - bx0) * 4096 + r * 128 +
               ((static_cast<uint32_t>((c % 32) >> 2) ^ rsw) << 4) + 4 * (c & 3);
      };
      if (p.accumulate && rows_in) {
        if (!load_previous_boxes(tmap_out, p, tc, quarter, lane, stage_out, oldout_bar, oldout_phase, abort_flag,
                                 PER_ROUND, 4096, [&](int b) { return col0 + (bx0 + b) * 32; }))
          return false;
#pragma unroll
        for (int f = 0; f < COLS; f += 2) {
          if (frag_col<GC>(f, 0) / 32 < bx0 || frag_col<GC>(f, 0) / 32 >= bx0 + PER_ROUND) continue;
          const uint2 w = ld_shared_v2(addr_of(f));
          fin[f] += __uint_as_float(w.x);
          fin[f + 1] += __uint_as_float(w.y);
        }
      }
#pragma unroll
      for (int f = 0; f < COLS; f += 2) {
        if (frag_col<GC>(f, 0) / 32 < bx0 || frag_col<GC>(f, 0) / 32 >= bx0 + PER_ROUND) continue;
        st_shared_v2(addr_of(f), __float_as_uint(fin[f]), __float_as_uint(fin[f + 1]));
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && rows_in) {
#pragma unroll
        for (int bi = 0; bi < PER_ROUND; ++bi) {
          const int c = col0 + (bx0 + bi) * 32;
          if (c < p.n) tma_store_3d(&tmap_out, stage_out + bi * 4096, c, tc.m0 + quarter * 32, tc.e);
        }
        bulk_commit_group();
      }
    }
  }
  return true;
}

// PAIR: a cluster of two CTAs computes a 256 x BN tile with cta_group::2
// UMMAs issued by the even CTA; each CTA loads its 128 rows of A and half of
// B (a third less operand traffic per SM than a 128 x BN tile) and promotes
// its own 128 TMEM lanes. The odd CTA's promotion warps release a partial on
// the even CTA's barrier.
template <int BN, int EPI, bool PAIR>
__global__ void __launch_bounds__(Cfg<BN, EPI, PAIR>::THREADS, Cfg<BN, EPI, PAIR>::CTAS_PER_SM)
    grouped_wgrad_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                         const __grid_constant__ CUtensorMap tmap_out, const GemmParams p) {
  using C = Cfg<BN, EPI, PAIR>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_a = smem;
  uint8_t* s_b = s_a + C::STAGES * C::A_BYTES;
  uint8_t* s_out = s_b + C::STAGES * C::B_BYTES;
  float* s_scale = reinterpret_cast<float*>(s_out + C::EPI_WARPS * C::OUT_STAGE_BYTES_PER_WARP);
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_scale + C::SSTAGES * C::SCALE_FLOATS);
  uint64_t* full_bar = bars;                          // [C::STAGES]   TMA -> MMA
  uint64_t* empty_bar = full_bar + C::STAGES;            // [C::STAGES]   MMA -> TMA
  uint64_t* sfull_bar = empty_bar + C::STAGES;           // [C::SSTAGES] TMA -> epilogue
  uint64_t* sempty_bar = sfull_bar + C::SSTAGES;    // [C::SSTAGES] epilogue -> TMA
  uint64_t* tfull_bar = sempty_bar + C::SSTAGES;    // [2] MMA -> epilogue
  uint64_t* tempty_bar = tfull_bar + 2;               // [2] epilogue -> MMA
  uint64_t* oldout_bar = tempty_bar + 2;             // [EPI_WARPS] previous output -> promotion warp (accumulate)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(oldout_bar + C::EPI_WARPS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int tile_begin = PAIR ? static_cast<int>(cluster_id_x()) : static_cast<int>(blockIdx.x);
  const int tile_stride = PAIR ? static_cast<int>(cluster_count_x()) : static_cast<int>(gridDim.x);
  const int row_off = static_cast<int>(rank) * BM;
#if WGRAD_PROFILE
  __shared__ unsigned long long s_prof[kProfSlots];
  __shared__ long long s_issue[8];
  const bool prof_lane = lane == 0 && (warp == 0 || warp == 1 || warp == FIRST_EPI_WARP);
  if (threadIdx.x < kProfSlots) s_prof[threadIdx.x] = threadIdx.x == kProfCtas ? 1ull : 0ull;
#endif

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::STAGES; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < C::SSTAGES; ++i) {
      mbar_init(&sfull_bar[i], 1);
      mbar_init(&sempty_bar[i], C::EPI_WARPS);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], (PAIR ? 2 : 1) * C::EPI_WARPS);  // a pair's even CTA hears both CTAs
    }
    for (int i = 0; i < C::EPI_WARPS; ++i) mbar_init(&oldout_bar[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0 && p.has_operands) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    tma_prefetch_desc(&tmap_out);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_holder, C::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_holder, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
#if WGRAD_PROFILE
  const long long t_cta0 = clock64();
#endif

  if (warp < FIRST_EPI_WARP) setmaxnreg_dec<C::REGS_CONTROL>();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0)
      run_producer<C, BN, PAIR>(tmap_a, tmap_b, p, s_a, s_b, s_scale, full_bar, empty_bar, sfull_bar, sempty_bar,
                                abort_flag, WGRAD_PROF_PTR, tile_begin, tile_stride, rank);
  } else if (warp == 1 && rank == 0) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = umma_idesc_e4m3_f32(PAIR ? 2 * BM : BM, BN);
    int trace_b = 0;
    int stage = 0, acc = 0;
    uint32_t phase = 0, aphase = 0;
    bool ok = true;
    for (int r = 0, tile = tile_begin; r * tile_stride < p.num_tiles && ok; tile = sched_tile<PAIR>(++r, tile_begin, tile_stride)) {
    if (tile >= p.num_tiles) continue;
      const TileCoord tc = decode_tile(p, tile);
      const int nkb = __ldg(p.block_offsets + tc.e + 1) - __ldg(p.block_offsets + tc.e);
      // K slices of 32 rows in the expert's last block: 4 in the padded layout;
      // in the packed layout only the slices that hold the expert's rows (the
      // rest of the 128-row TMA box belongs to the next expert or the guard).
      const int klen = __ldg(p.k_row_offsets + tc.e + 1) - __ldg(p.k_row_offsets + tc.e);
      const int last_atoms = min(4, max(1, (klen - (nkb - 1) * BK + 31) / 32));
      for (int kb = 0; kb < nkb; ++kb, ++trace_b) {
        const int atoms = kb + 1 == nkb ? last_atoms : BK / 32;
        // Whole warp waits (keeps the warp converged for the .sync.aligned ops).
        WGRAD_PROF_T(tm0);
        ok = mbar_wait2(&tempty_bar[acc], aphase ^ 1u, &full_bar[stage], phase, abort_flag, kDevTimeoutMma);
        WGRAD_PROF_ADD(kProfMmaWait, tm0);
        WGRAD_PROF_LATENCY(stage);
        WGRAD_PROF_T(tm1);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
#if WGRAD_TRACE == 1
        WGRAD_TRACE_EV(kTrMmaReady, trace_b);
#endif
        tc_fence_after();
        if (elect_one_sync()) {
          const uint32_t a_addr = smem_u32(s_a + stage * C::A_BYTES);
          const uint32_t b_addr = smem_u32(s_b + stage * C::B_BYTES);
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            if (k >= atoms) break;
            // advance 32 bytes (one K=32 FP8 slice) inside the 128-byte swizzle atom
            if constexpr (PAIR) {
              umma_f8_pair(d_tmem, umma_desc_k_sw128(a_addr + k * 32), umma_desc_k_sw128(b_addr + k * 32), idesc,
                           k > 0 ? 1u : 0u);
            } else {
              umma_f8(d_tmem, umma_desc_k_sw128(a_addr + k * 32), umma_desc_k_sw128(b_addr + k * 32), idesc,
                      k > 0 ? 1u : 0u);
            }
          }
          if constexpr (PAIR) {  // release the stage and publish the partial in both CTAs
            umma_commit_pair(cluster_addr(&empty_bar[stage], 0));
            umma_commit_pair(cluster_addr(&empty_bar[stage], 1));
            umma_commit_pair(cluster_addr(&tfull_bar[acc], 0));
            umma_commit_pair(cluster_addr(&tfull_bar[acc], 1));
          } else {
            umma_commit(&empty_bar[stage]);
            umma_commit(&tfull_bar[acc]);
          }
        }
        __syncwarp();
#if WGRAD_TRACE == 1
        WGRAD_TRACE_EV(kTrMmaIssued, trace_b);
#endif
        WGRAD_PROF_ADD(kProfMmaIssue, tm1);
        if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        acc ^= 1;
        if (acc == 0) aphase ^= 1u;
      }
    }
  } else if (warp >= FIRST_EPI_WARP) {
    // ------------------------------------------------------------ promotion + epilogue
    setmaxnreg_inc<C::REGS_EPILOGUE>();
    const int ew = warp - FIRST_EPI_WARP;    // 0 .. EPI_WARPS-1
    const int quarter = warp & 3;            // TMEM lane quarter this warp may access
    const int half = ew >> 2;                // column group of the tile
    const int row = quarter * 32 + lane;     // row within the tile == TMEM lane
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    uint8_t* stage_out = s_out + ew * C::OUT_STAGE_BYTES_PER_WARP;

    int acc = 0, sstage = 0;
    uint32_t aphase = 0, sphase = 0, oldout_phase = 0;
    bool ok = true;
    // the partial's release goes to the pair's even CTA
    const uint32_t tempty_addr0 = PAIR ? cluster_addr(&tempty_bar[0], 0) : 0u;
    int trace_b = 0;
    for (int r = 0, tile = tile_begin; r * tile_stride < p.num_tiles && ok; tile = sched_tile<PAIR>(++r, tile_begin, tile_stride)) {
    if (tile >= p.num_tiles) continue;
      // trace 1: tile start and tile decoded, in the slots the scale-product kernel uses for its second half
      if (ew == 0 && WGRAD_TRACE == 1) WGRAD_TRACE_EV(kTrMmaHalfReady, trace_b);
      const TileCoord tc = decode_tile(p, tile, row_off);
      const int nkb = __ldg(p.block_offsets + tc.e + 1) - __ldg(p.block_offsets + tc.e);
      float fin[C::COLS_PER_WARP];
#pragma unroll
      for (int j = 0; j < C::COLS_PER_WARP; ++j) fin[j] = 0.f;
      if (ew == 0 && WGRAD_TRACE == 1 && nkb > 0) WGRAD_TRACE_EV(kTrMmaHalfIssued, trace_b);

      for (int kb = 0; kb < nkb; ++kb, ++trace_b) {
        if (ew == 0) WGRAD_TRACE_EV(WGRAD_TRACE == 2 ? 7 : kTrEpiWaitStart, trace_b);
        WGRAD_PROF_T(te0);
        ok = mbar_wait2(&tfull_bar[acc], aphase, &sfull_bar[sstage], sphase, abort_flag, kDevTimeoutEpilogue);
        WGRAD_PROF_ADD(kProfEpiWait, te0);
        WGRAD_PROF_T(te1);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        if (ew == 0) WGRAD_TRACE_EV(WGRAD_TRACE == 2 ? 0 : kTrEpiReady, trace_b);
        tc_fence_after();
        const float* sc = s_scale + sstage * C::SCALE_FLOATS;
#if WGRAD_DEBUG_MODES
        const bool unit_scales = p.mode == kModeUnscaled;  // raw FP8 product only
        const bool unit_raw = p.mode == kModeScaleOnly;    // scale product only
        const float a_s = unit_scales ? 1.f : sc[row];
#else
        const float a_s = sc[row];
#endif
        const float* b_s = sc + BM + half * C::COLS_PER_WARP;
        const uint32_t t_addr = tmem_base + lane_addr + static_cast<uint32_t>(acc * BN + half * C::COLS_PER_WARP);
        // Software pipeline over 32-column chunks: the TMEM load of chunk c+1
        // is in flight while chunk c is promoted. Once the last chunk is in
        // registers the TMEM buffer goes back to the MMA warp, before its math.
        constexpr int CH = C::CHUNK;
        if constexpr (C::FRAG16) {
          // Chunk c: 8-column groups [c GC, (c + 1) GC) of both 16-row halves of
          // the warp's lanes, one load per half, one wait; the chunk's column
          // scales are one 8-byte load per group, shared by both halves.
          constexpr int GC = C::GC;
          constexpr int NCH = C::COLS_PER_WARP / (8 * GC);
          static_assert(GC == 4 || GC == 2, "one 16x256b.x4 or .x2 load per half per chunk");
          const int rq = lane >> 2;
#if WGRAD_DEBUG_MODES
          const float sa4[4] = {unit_scales ? 1.f : sc[quarter * 32 + rq], unit_scales ? 1.f : sc[quarter * 32 + rq + 8],
                                unit_scales ? 1.f : sc[quarter * 32 + rq + 16],
                                unit_scales ? 1.f : sc[quarter * 32 + rq + 24]};
#else
          const float sa4[4] = {sc[quarter * 32 + rq], sc[quarter * 32 + rq + 8], sc[quarter * 32 + rq + 16],
                                sc[quarter * 32 + rq + 24]};
#endif
          const float* sb_t = b_s + 2 * (lane & 3);
          uint32_t r[2][8 * GC];
          auto ld_half = [](uint32_t addr, uint32_t* dst) {
            if constexpr (GC == 4) tmem_ld_16x256b_x4(addr, dst);
            else tmem_ld_16x256b_x2(addr, dst);
          };
          ld_half(t_addr, r[0]);
          ld_half(t_addr + (16u << 16), r[0] + 4 * GC);
#pragma unroll
          for (int c = 0; c < NCH; ++c) {
            tmem_wait_ld_bind(r[c & 1]);
#if WGRAD_TRACE == 2
            if (ew == 0 && c < 4) WGRAD_TRACE_EV(1 + c, trace_b);
#endif
            if (c + 1 < NCH) {
              ld_half(t_addr + (c + 1) * 8 * GC, r[(c + 1) & 1]);
              ld_half(t_addr + (16u << 16) + (c + 1) * 8 * GC, r[(c + 1) & 1] + 4 * GC);
            } else {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) {
                if (PAIR && rank != 0) mbar_arrive_cluster(tempty_addr0 + static_cast<uint32_t>(acc * sizeof(uint64_t)));
                else mbar_arrive(&tempty_bar[acc]);
              }
              if (ew == 0) WGRAD_TRACE_EV(WGRAD_TRACE == 2 ? 5 : kTrEpiReleased, trace_b);
            }
#pragma unroll
            for (int g = 0; g < GC; ++g) {
#if WGRAD_DEBUG_MODES
              const float2 sb2 = unit_scales ? make_float2(1.f, 1.f)
                                             : *reinterpret_cast<const float2*>(sb_t + 8 * (c * GC + g));
#else
              const float2 sb2 = *reinterpret_cast<const float2*>(sb_t + 8 * (c * GC + g));
#endif
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const uint32_t* q = &r[c & 1][h * 4 * GC + 4 * g];
                float* f = &fin[c * 8 * GC + h * 4 * GC + 4 * g];
#if WGRAD_DEBUG_MODES
                const uint32_t one = __float_as_uint(1.f);
                const float q0 = __uint_as_float(unit_raw ? one : q[0]), q1 = __uint_as_float(unit_raw ? one : q[1]);
                const float q2 = __uint_as_float(unit_raw ? one : q[2]), q3 = __uint_as_float(unit_raw ? one : q[3]);
#else
                const float q0 = __uint_as_float(q[0]), q1 = __uint_as_float(q[1]);
                const float q2 = __uint_as_float(q[2]), q3 = __uint_as_float(q[3]);
#endif
                float u0, u1, u2, u3;
                mul_f32x2(u0, u1, q0, q1, sb2.x, sb2.y);
                mul_f32x2(u2, u3, q2, q3, sb2.x, sb2.y);
                fma_f32x2(f[0], f[1], u0, u1, sa4[2 * h], sa4[2 * h], f[0], f[1]);
                fma_f32x2(f[2], f[3], u2, u3, sa4[2 * h + 1], sa4[2 * h + 1], f[2], f[3]);
              }
            }
          }
        } else {
          uint32_t r[2][CH];
          tmem_ld_chunk(t_addr, r[0]);
#pragma unroll
          for (int c = 0; c < C::CHUNKS; ++c) {
            tmem_wait_ld_bind(r[c & 1]);
#if WGRAD_TRACE == 2
            if (ew == 0 && c < 4) WGRAD_TRACE_EV(1 + c, trace_b);
#endif
            if (c + 1 < C::CHUNKS) {
              tmem_ld_chunk(t_addr + (c + 1) * CH, r[(c + 1) & 1]);
            } else {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) {
                if (PAIR && rank != 0) mbar_arrive_cluster(tempty_addr0 + static_cast<uint32_t>(acc * sizeof(uint64_t)));
                else mbar_arrive(&tempty_bar[acc]);
              }
              if (ew == 0) WGRAD_TRACE_EV(WGRAD_TRACE == 2 ? 5 : kTrEpiReleased, trace_b);
            }
#pragma unroll
            for (int j = 0; j < CH; j += 4) {
#if WGRAD_DEBUG_MODES
              const float4 sb4 = unit_scales ? make_float4(1.f, 1.f, 1.f, 1.f)
                                             : *reinterpret_cast<const float4*>(b_s + c * CH + j);
              const uint32_t one = __float_as_uint(1.f);
              const uint32_t q[4] = {unit_raw ? one : r[c & 1][j], unit_raw ? one : r[c & 1][j + 1],
                                     unit_raw ? one : r[c & 1][j + 2], unit_raw ? one : r[c & 1][j + 3]};
#else
              const float4 sb4 = *reinterpret_cast<const float4*>(b_s + c * CH + j);
              const uint32_t* q = &r[c & 1][j];
#endif
              float u0, u1, u2, u3;
              mul_f32x2(u0, u1, __uint_as_float(q[0]), __uint_as_float(q[1]), sb4.x, sb4.y);
              mul_f32x2(u2, u3, __uint_as_float(q[2]), __uint_as_float(q[3]), sb4.z, sb4.w);
              float* f = &fin[c * CH + j];
              fma_f32x2(f[0], f[1], u0, u1, a_s, a_s, f[0], f[1]);
              fma_f32x2(f[2], f[3], u2, u3, a_s, a_s, f[2], f[3]);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sempty_bar[sstage]);
        if (ew == 0) WGRAD_TRACE_EV(WGRAD_TRACE == 2 ? 6 : kTrEpiDone, trace_b);
        WGRAD_PROF_ADD(kProfEpiPromote, te1);
        WGRAD_PROF_INC(kProfKBlocks);
        acc ^= 1;
        if (acc == 0) aphase ^= 1u;
        if (++sstage == C::SSTAGES) { sstage = 0; sphase ^= 1u; }
      }
      if (!ok) break;

      // -------------------------------------------------------- epilogue store
      WGRAD_PROF_T(ts0);
      WGRAD_PROF_INC(kProfTiles);
      const int col0 = tc.n0 + half * C::COLS_PER_WARP;
#if WGRAD_DEBUG_MODES
      const int g_row = tc.m0 + row;
      if (p.mode == kModeCoordM || p.mode == kModeCoordN || p.mode == kModeScaleOnly) {
#pragma unroll
        for (int j = 0; j < C::COLS_PER_WARP; ++j) {
          const int jr = C::FRAG16 ? tc.m0 + quarter * 32 + frag_row<C::GC>(j, lane) : g_row;
          const int jc = C::FRAG16 ? frag_col<C::GC>(j, lane) : j;
          fin[j] = p.mode == kModeCoordM ? static_cast<float>(jr)
                 : p.mode == kModeCoordN ? static_cast<float>(col0 + jc)
                                         : fin[j] * 1048576.0f;  // 2^20, as the reference
        }
      }
#endif
      // The previous tile's TMA store must have finished reading the staging buffer.
      WGRAD_PROF_T(ts1);
      if (lane == 0) bulk_wait_group_read0();
      __syncwarp();
      WGRAD_PROF_ADD(kProfEpiStoreWait, ts1);
      if constexpr (C::FRAG16)
        ok = store_warp_tile_frag<C::COLS_PER_WARP, C::OUT_STAGE_BYTES_PER_WARP, C::GC>(
            fin, tmap_out, p, tc, quarter, lane, col0, stage_out, &oldout_bar[ew], oldout_phase, abort_flag);
      else
        ok = store_warp_tile<C::COLS_PER_WARP, C::OUT_STAGE_BYTES_PER_WARP>(
            fin, tmap_out, p, tc, quarter, lane, col0, stage_out, &oldout_bar[ew], oldout_phase, abort_flag);
      if (!ok) break;
      WGRAD_PROF_ADD(kProfEpiStore, ts0);
    }
    if (lane == 0) bulk_wait_group0();  // all output writes complete before exit
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // no cross-CTA arrival or UMMA is left in flight
#if WGRAD_PROFILE
  if (threadIdx.x < kProfSlots)
    atomicAdd(&g_wgrad_prof[threadIdx.x], threadIdx.x == kProfCtaCycles
                                              ? static_cast<unsigned long long>(clock64() - t_cta0)
                                              : s_prof[threadIdx.x]);
#endif
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    else tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}


// ---------------------------------------------------------------------------
// UE8M0 variant: scales that are powers of two are applied by the tensor core
// (tcgen05.mma kind::mxf8f6f4.block_scale, one E8M0 scale per row of A / B
// and 32-wide K slice), so a tile's K blocks accumulate in one TMEM buffer and
// no fp32 promotion runs. Exact for such scales: the sum is the same
// sum_b sum_k qa qb sa sb, rounded once per UMMA instead of once per K block.
//
// Warps: 0 TMA producer (shared with the promotion kernel), 1 MMA issuer,
// 2 scale-factor writer, 4..15 epilogue (three 64-column warps per TMEM lane
// quarter). Per K block the writer turns the block's fp32 scales into E8M0
// bytes in shared memory, in the 32-row x 16-byte layout of the CUTLASS Sm1xx
// block-scaled atom: row r of A or B at byte 16 (r % 32) + 4 (r / 32 % 4) + j
// of its 128-row group, j the K slice. The MMA thread copies them into TMEM
// with tcgen05.cp 32x128b.warpx4 (row r -> lane r % 32 of every quarter,
// column r / 32), in order with its UMMAs. TMEM: two 192-column accumulators,
// then SF_STAGES scale-factor stages of 16 columns (A: 4, B: 8 from +4). The
// four K slices of a 128-row block share one scale, so all four bytes of a
// word are equal and the instruction's byte selectors stay 0.
struct BsCfg {
  static constexpr int BN = 192;
  static constexpr int STAGES = 4;
  static constexpr int SF_WARP = 2;
  static constexpr int FIRST_EPI = 4;
  static constexpr int EPI_WARPS = 12;
  static constexpr int THREADS = 32 * (FIRST_EPI + EPI_WARPS);
  static constexpr int COLS_PER_WARP = BN / (EPI_WARPS / 4);  // 64
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int SCALE_FLOATS = BM + BN;
  static constexpr int SSTAGES = 6;  // scale-vector ring depth
  static constexpr int OUT_STAGE_BYTES_PER_WARP = 4096;
  static constexpr int SF_STAGES = 4;
  static constexpr int SF_A_BYTES = 512;    // 128 rows
  static constexpr int SF_B_BYTES = 1024;   // 256 rows (BN = 192 uses 6 of the 8 columns)
  static constexpr int SF_STAGE_BYTES = SF_A_BYTES + SF_B_BYTES;
  static constexpr int SF_COL0 = 2 * BN;
  static constexpr int SF_STAGE_COLS = 16;
  static constexpr int SF_B_OFFSET = 4;
  static constexpr int TMEM_COLS = 512;
  static constexpr int SMEM_BYTES = STAGES * (A_BYTES + B_BYTES) + EPI_WARPS * OUT_STAGE_BYTES_PER_WARP +
                                    SF_STAGES * SF_STAGE_BYTES + SSTAGES * SCALE_FLOATS * 4 +
                                    512 /*barriers*/ + 1024 /*align*/;
  static_assert(SF_COL0 + SF_STAGES * SF_STAGE_COLS <= TMEM_COLS, "TMEM columns");
  static_assert(COLS_PER_WARP * 32 * 2 == OUT_STAGE_BYTES_PER_WARP, "one BF16 staging round per tile");
  static_assert(SMEM_BYTES <= 232448, "shared memory");
};

// E8M0 byte of a positive power-of-two fp32 scale, replicated into the four
// bytes of a word; anything else (mantissa bits, zero, subnormal, inf, NaN,
// negative) encodes as 1.0 and sets `bad` (the caller records device error 6).
// Branch-free, so a warp's scale loads can all be in flight together.
__device__ __forceinline__ uint32_t e8m0_word(float s, bool& bad) {
  const uint32_t bits = __float_as_uint(s);
  const uint32_t e = bits >> 23;  // sign bit set -> e > 255
  const bool invalid = (bits & 0x7FFFFFu) != 0u || e == 0u || e >= 255u;
  bad |= invalid;
  return (invalid ? 127u : e) * 0x01010101u;
}

__global__ void __launch_bounds__(BsCfg::THREADS, 1)
    grouped_wgrad_ue8m0_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                               const __grid_constant__ CUtensorMap tmap_out, const GemmParams p) {
  using C = BsCfg;
  constexpr int BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_a = smem;
  uint8_t* s_b = s_a + C::STAGES * C::A_BYTES;
  uint8_t* s_out = s_b + C::STAGES * C::B_BYTES;
  uint8_t* s_sf = s_out + C::EPI_WARPS * C::OUT_STAGE_BYTES_PER_WARP;    // [SF_STAGES][A 512 | B 1024]
  float* s_scale = reinterpret_cast<float*>(s_sf + C::SF_STAGES * C::SF_STAGE_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_scale + C::SSTAGES * C::SCALE_FLOATS);
  uint64_t* full_bar = bars;                             // [STAGES]      TMA -> MMA
  uint64_t* empty_bar = full_bar + C::STAGES;            // [STAGES]      MMA -> TMA
  uint64_t* sfull_bar = empty_bar + C::STAGES;           // [C::SSTAGES] TMA -> SF writer
  uint64_t* sempty_bar = sfull_bar + C::SSTAGES;       // [C::SSTAGES] SF writer -> TMA
  uint64_t* sffull_bar = sempty_bar + C::SSTAGES;      // [SF_STAGES]   SF writer -> MMA
  uint64_t* sfempty_bar = sffull_bar + C::SF_STAGES;     // [SF_STAGES]   MMA (copies done) -> SF writer
  uint64_t* tfull_bar = sfempty_bar + C::SF_STAGES;      // [2] MMA -> epilogue
  uint64_t* tempty_bar = tfull_bar + 2;                  // [2] epilogue -> MMA
  uint64_t* oldout_bar = tempty_bar + 2;                 // [EPI_WARPS] previous output (accumulate)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(oldout_bar + C::EPI_WARPS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
#if WGRAD_PROFILE
  // Slots as the promotion kernel: MmaWait = operand + scale-factor stage,
  // EpiWait / EpiPromote = scale-factor writer wait / work, EpiStoreWait =
  // epilogue wait for the accumulator, EpiStore = its drain + store.
  __shared__ unsigned long long s_prof[kProfSlots];
  __shared__ long long s_issue[8];
  const bool prof_lane = lane == 0 && (warp == 0 || warp == 1 || warp == BsCfg::SF_WARP || warp == BsCfg::FIRST_EPI);
  if (threadIdx.x < kProfSlots) s_prof[threadIdx.x] = threadIdx.x == kProfCtas ? 1ull : 0ull;
#endif

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::STAGES; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < C::SSTAGES; ++i) {
      mbar_init(&sfull_bar[i], 1);
      mbar_init(&sempty_bar[i], 1);
    }
    for (int i = 0; i < C::SF_STAGES; ++i) {
      mbar_init(&sffull_bar[i], 1);
      mbar_init(&sfempty_bar[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], C::EPI_WARPS);
    }
    for (int i = 0; i < C::EPI_WARPS; ++i) mbar_init(&oldout_bar[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0 && p.has_operands) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    tma_prefetch_desc(&tmap_out);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
#if WGRAD_PROFILE
  const long long t_cta0 = clock64();
#endif

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) run_producer<C, BN>(tmap_a, tmap_b, p, s_a, s_b, s_scale, full_bar, empty_bar, sfull_bar, sempty_bar,
                                       abort_flag, WGRAD_PROF_PTR);
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = umma_idesc_mxf8_e4m3_ue8m0(BM, BN);
    int stage = 0, sfs = 0, acc = 0;
    uint32_t phase = 0, sfphase = 0, aphase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
      const TileCoord tc = decode_tile(p, tile);
      const int nkb = __ldg(p.block_offsets + tc.e + 1) - __ldg(p.block_offsets + tc.e);
      if (nkb == 0) continue;  // empty expert: the epilogue writes zeros without the accumulator
      const int klen = __ldg(p.k_row_offsets + tc.e + 1) - __ldg(p.k_row_offsets + tc.e);
      const int last_atoms = min(4, max(1, (klen - (nkb - 1) * BK + 31) / 32));
      WGRAD_PROF_T(tt0);
      ok = mbar_wait(&tempty_bar[acc], aphase ^ 1u, abort_flag, kDevTimeoutMma);
      WGRAD_PROF_ADD(kProfMmaTileWait, tt0);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
      for (int kb = 0; kb < nkb; ++kb) {
        const int atoms = kb + 1 == nkb ? last_atoms : BK / 32;
        WGRAD_PROF_T(tm0);
        ok = mbar_wait2(&full_bar[stage], phase, &sffull_bar[sfs], sfphase, abort_flag, kDevTimeoutMma);
        WGRAD_PROF_ADD(kProfMmaWait, tm0);
        WGRAD_PROF_LATENCY(stage);
        WGRAD_PROF_T(tm1);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        if (elect_one_sync()) {
          const uint32_t a_addr = smem_u32(s_a + stage * C::A_BYTES);
          const uint32_t b_addr = smem_u32(s_b + stage * C::B_BYTES);
          const uint32_t sf_smem = smem_u32(s_sf + sfs * C::SF_STAGE_BYTES);
          const uint32_t sfa = tmem_base + static_cast<uint32_t>(C::SF_COL0 + sfs * C::SF_STAGE_COLS);
          tmem_cp_32x128b_warpx4(sfa, smem_desc_rows16(sf_smem));
          tmem_cp_32x128b_warpx4(sfa + C::SF_B_OFFSET, smem_desc_rows16(sf_smem + C::SF_A_BYTES));
          tmem_cp_32x128b_warpx4(sfa + C::SF_B_OFFSET + 4, smem_desc_rows16(sf_smem + C::SF_A_BYTES + 512));
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            if (k >= atoms) break;
            umma_mxf8(d_tmem, umma_desc_k_sw128(a_addr + k * 32), umma_desc_k_sw128(b_addr + k * 32), idesc, sfa,
                      sfa + C::SF_B_OFFSET, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          umma_commit(&sfempty_bar[sfs]);
        }
        __syncwarp();
        WGRAD_PROF_ADD(kProfMmaIssue, tm1);
        if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        if (++sfs == C::SF_STAGES) { sfs = 0; sfphase ^= 1u; }
      }
      if (!ok) break;
      if (elect_one_sync()) umma_commit(&tfull_bar[acc]);
      __syncwarp();
      acc ^= 1;
      if (acc == 0) aphase ^= 1u;
    }
  } else if (warp == C::SF_WARP) {
    // ------------------------------------------------------------ scale-factor writer
    int sstage = 0, sfs = 0;
    uint32_t sphase = 0, sfphase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
      const TileCoord tc = decode_tile(p, tile);
      const int nkb = __ldg(p.block_offsets + tc.e + 1) - __ldg(p.block_offsets + tc.e);
      const int a_valid = min(BM, p.m - tc.m0);
      const int b_valid = min(BN, p.n - tc.n0);
      for (int kb = 0; kb < nkb; ++kb) {
        WGRAD_PROF_T(tf0);
        ok = mbar_wait2(&sfull_bar[sstage], sphase, &sfempty_bar[sfs], sfphase ^ 1u, abort_flag, kDevTimeoutEpilogue);
        WGRAD_PROF_ADD(kProfEpiWait, tf0);
        WGRAD_PROF_T(tf1);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        WGRAD_PROF_ADD(kProfSfSync, tf1);
        WGRAD_PROF_T(tf3);
        const float* sc = s_scale + sstage * C::SCALE_FLOATS;
        // A rows lane + 32 c (c < 4), then B rows lane + 32 (c - 4); rows past the
        // operand's edge read as 1.0. All twelve loads first, then the conversion.
        float v[12];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int r = lane + 32 * c;
          v[c] = r < a_valid ? sc[r] : 1.0f;
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int r = lane + 32 * c;
          v[4 + c] = (r < BN && r < b_valid) ? sc[BM + r] : 1.0f;
        }
        uint32_t w[12];
        bool bad = false;
#pragma unroll
        for (int c = 0; c < 12; ++c) w[c] = e8m0_word(v[c], bad);
        if (bad) record_device_error(kDevScaleNotPow2);
#if WGRAD_PROFILE
#pragma unroll
        for (int i = 0; i < 12; ++i) asm volatile("" ::"r"(w[i]));  // the loads have landed
        WGRAD_PROF_ADD(kProfSfLoad, tf3);
#endif
        const uint32_t dst = smem_u32(s_sf + sfs * C::SF_STAGE_BYTES) + lane * 16;
        st_shared_v4(dst, w[0], w[1], w[2], w[3]);
        st_shared_v4(dst + C::SF_A_BYTES, w[4], w[5], w[6], w[7]);
        st_shared_v4(dst + C::SF_A_BYTES + 512, w[8], w[9], w[10], w[11]);
        WGRAD_PROF_ADD(kProfSfConvert, tf1);
        WGRAD_PROF_T(tf2);
        fence_proxy_async_smem();  // the copies read through the async proxy
        __syncwarp();
        if (elect_one_sync()) {
          mbar_arrive(&sempty_bar[sstage]);
          mbar_arrive(&sffull_bar[sfs]);
        }
        WGRAD_PROF_ADD(kProfSfPublish, tf2);
        WGRAD_PROF_ADD(kProfEpiPromote, tf1);
        WGRAD_PROF_INC(kProfKBlocks);
        if (++sstage == C::SSTAGES) { sstage = 0; sphase ^= 1u; }
        if (++sfs == C::SF_STAGES) { sfs = 0; sfphase ^= 1u; }
      }
    }
  } else if (warp >= C::FIRST_EPI) {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - C::FIRST_EPI;   // 0 .. EPI_WARPS-1
    const int quarter = warp & 3;
    const int cgroup = ew >> 2;           // 64-column group of the tile
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    uint8_t* stage_out = s_out + ew * C::OUT_STAGE_BYTES_PER_WARP;
    int acc = 0;
    uint32_t aphase = 0, oldout_phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
      const TileCoord tc = decode_tile(p, tile);
      const int nkb = __ldg(p.block_offsets + tc.e + 1) - __ldg(p.block_offsets + tc.e);
      float fin[C::COLS_PER_WARP];
      if (nkb == 0) {
#pragma unroll
        for (int j = 0; j < C::COLS_PER_WARP; ++j) fin[j] = 0.f;
      } else {
        WGRAD_PROF_T(te0);
        ok = mbar_wait(&tfull_bar[acc], aphase, abort_flag, kDevTimeoutEpilogue);
        WGRAD_PROF_ADD(kProfEpiStoreWait, te0);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        const uint32_t t_addr =
            tmem_base + lane_addr + static_cast<uint32_t>(acc * BN + cgroup * C::COLS_PER_WARP);
        uint32_t r0[32], r1[32];
        tmem_ld_32x32b_x32(t_addr, r0);
        tmem_ld_32x32b_x32(t_addr + 32, r1);
        tmem_wait_ld_bind(r0);
        tmem_wait_ld_bind(r1);
        tc_fence_before();
        __syncwarp();
        if (elect_one_sync()) mbar_arrive(&tempty_bar[acc]);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          fin[j] = __uint_as_float(r0[j]);
          fin[32 + j] = __uint_as_float(r1[j]);
        }
        acc ^= 1;
        if (acc == 0) aphase ^= 1u;
      }
      const int col0 = tc.n0 + cgroup * C::COLS_PER_WARP;
      WGRAD_PROF_T(ts0);
      WGRAD_PROF_INC(kProfTiles);
      // The previous tile's TMA store must have finished reading the staging buffer.
      if (lane == 0) bulk_wait_group_read0();
      __syncwarp();
      ok = store_warp_tile<C::COLS_PER_WARP, C::OUT_STAGE_BYTES_PER_WARP>(
          fin, tmap_out, p, tc, quarter, lane, col0, stage_out, &oldout_bar[ew], oldout_phase, abort_flag);
      WGRAD_PROF_ADD(kProfEpiStore, ts0);
    }
    if (lane == 0) bulk_wait_group0();  // all output writes complete before exit
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
#if WGRAD_PROFILE
  if (threadIdx.x < kProfSlots)
    atomicAdd(&g_wgrad_prof[threadIdx.x], threadIdx.x == kProfCtaCycles
                                              ? static_cast<unsigned long long>(clock64() - t_cta0)
                                              : s_prof[threadIdx.x]);
#endif
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace

// Raises a kernel's dynamic shared-memory limit once per (kernel, device);
// thread-safe (a std::once_flag per device ordinal), and every later call on
// that device returns the first attempt's result.
template <auto Kernel>
static cudaError_t configure_once(int smem_bytes) {
  static std::once_flag flags[kMaxDevices];
  static cudaError_t result[kMaxDevices];
  int dev = 0;
  const cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::call_once(flags[dev], [&] {
    result[dev] = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
  });
  return result[dev];
}

template <int BN, int EPI, bool PAIR = false>
static cudaError_t launch_impl(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                               const GemmParams& p, int grid, cudaStream_t stream) {
  using C = Cfg<BN, EPI, PAIR>;
  const cudaError_t err = configure_once<grouped_wgrad_kernel<BN, EPI, PAIR>>(C::SMEM_BYTES);
  if (err != cudaSuccess) return err;
  if constexpr (PAIR) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(grid & ~1));  // whole clusters of two
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, grouped_wgrad_kernel<BN, EPI, PAIR>, ta, tb, to, p);
  }
  grouped_wgrad_kernel<BN, EPI, PAIR><<<grid, C::THREADS, C::SMEM_BYTES, stream>>>(ta, tb, to, p);
  return cudaGetLastError();
}

static cudaError_t launch_ue8m0(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                                const GemmParams& p, int grid, cudaStream_t stream) {
  const cudaError_t err = configure_once<grouped_wgrad_ue8m0_kernel>(BsCfg::SMEM_BYTES);
  if (err != cudaSuccess) return err;
  grouped_wgrad_ue8m0_kernel<<<grid, BsCfg::THREADS, BsCfg::SMEM_BYTES, stream>>>(ta, tb, to, p);
  return cudaGetLastError();
}

cudaError_t launch_grouped_wgrad(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                                 const GemmParams& p, int grid, cudaStream_t stream) {
  if (p.ue8m0) return p.bn == BsCfg::BN ? launch_ue8m0(ta, tb, to, p, grid, stream) : cudaErrorInvalidValue;
  if (p.bm == 256) {
    if (p.bn != 256) return cudaErrorInvalidValue;
    return p.epi_warps == 16 ? launch_impl<256, 16, true>(ta, tb, to, p, grid, stream)
                             : launch_impl<256, 8, true>(ta, tb, to, p, grid, stream);
  }
  if (p.bn == 256) {
    return p.epi_warps == 16 ? launch_impl<256, 16>(ta, tb, to, p, grid, stream)
                             : launch_impl<256, 8>(ta, tb, to, p, grid, stream);
  }
  if (p.bn == 192) return launch_impl<192, 12>(ta, tb, to, p, grid, stream);
  return p.epi_warps == 4 ? launch_impl<128, 4>(ta, tb, to, p, grid, stream)
                          : launch_impl<128, 8>(ta, tb, to, p, grid, stream);
}

}  // namespace wgrad
