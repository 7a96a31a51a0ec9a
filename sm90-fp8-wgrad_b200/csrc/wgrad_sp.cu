// Grouped FP8 Wgrad on a CTA pair with the per-block scale product computed
// by the tensor core ("SP" kernel, tile config SM100_WGRAD_TILE_256x256_SP).
//
// Same math as grouped_wgrad_kernel (wgrad_gemm.cu) and the reference kernel
// Fp8ScaledWgradSm90 (src/sm90_fp8_wgrad/gemm_sm90.py:1211-2321):
//   out[e, m, n] = sum_b  sa[b, m] * sb[b, n] * P_b[m, n],
//   P_b[m, n]    = sum_{k in block b} A[m, k] * B[n, k]        (FP8 x FP8 -> fp32)
// but the rank-1 scale product S_b[m, n] = sa[b, m] * sb[b, n] that the
// reference's promotion (promote_scaled_acc_epilogue_staged, :5023-5085)
// multiplies in with two fp32 operations per element is produced by a
// kind::tf32 UMMA beside the FP8 partial, so the promotion is a single fused
// multiply-add per element:  fin = fma(P_b, S_b, fin).
//
// On B200 the two fp32 operations per element per 128-row K block take exactly
// as many FMA-pipe cycles as the block's FP8 UMMAs take tensor cycles, so the
// two-operation promotion cannot hide behind the tensor pipe. One K=8 TF32
// UMMA per 128 x 128 half tile (64 tensor cycles per SM, a quarter of the FP8
// block's 256) halves that work and leaves the FMA pipe slack.
//
// Scale product accuracy: every scale s is split as s = hi + lo with hi = s
// truncated to TF32 (11 significant bits) and lo = (s - hi) truncated to TF32;
// the K = 8 TF32 operand rows are A: [hi, hi, lo, lo, 0, 0, 0, 0] and
// B: [hi, lo, hi, lo, 0, 0, 0, 0], so the UMMA sums the four exact 22-bit
// products hi*hi + hi*lo + lo*hi + lo*lo in fp32. The relative error of S is
// below 2^-19 (the truncated parts of the two lo terms), far under the BF16
// output rounding (2^-9); fp32 outputs keep ~19 correct bits per block term.
//
// Layout per CTA pair (cluster of two CTAs on neighbouring SMs), tile 256 x 256:
//   * each CTA loads its 128 rows of A, and B as two 64-row boxes (its half of
//     each 128-column half of the tile), plus the TF32 scale operands: 128 rows
//     of the A side and 2 x 64 rows of the B side, 16 B each from global
//     (the split scales, written by scale_operand_kernel), 32 B each in shared
//     memory (TMA zero-fills the four K elements past the 16-byte row).
//   * the even CTA's MMA thread issues, per K block and half h (128 columns):
//     4 x tcgen05.mma.cta_group::2.kind::f8f6f4 (M 256, N 128, K 32) into the
//     P columns of TMEM slot h, and 1 x tcgen05.mma.cta_group::2.kind::tf32
//     (M 256, N 128, K 8) into its S columns; TMEM slot h = columns
//     [256 h, 256 h + 128) for P and [256 h + 128, 256 h + 256) for S.
//   * 8 promotion warps per CTA: warp w covers TMEM lane quarter w % 4 and the
//     64-column group (w / 4) of each half; it reads P and S of a half with
//     tcgen05.ld, hands the slot back, and accumulates fin = fma(P, S, fin) in
//     registers (128 columns per thread). At tile end: BF16 (or fp32) staging
//     and TMA stores, as the other kernels.
// Tile order: clusters walk the (LPT expert, m, n) tile list in a boustrophedon
// order (round r takes tiles r C + c, or r C + C - 1 - c on odd rounds), which
// evens out rounds of tiles sorted by descending K.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "ptx.cuh"
#include "wgrad_gemm.cuh"

namespace wgrad {

namespace {

constexpr int SP_CHUNK = 16;  // TMEM columns of P (and of S) per tcgen05.ld round trip

template <int EPI>
struct SpCfg {
  static constexpr int BM = 128;            // rows per CTA (256 per pair)
  static constexpr int BN = 256;            // columns per tile
  static constexpr int HALF = 128;          // columns per TMEM slot (UMMA N)
  static constexpr int BK = 128;            // K block = scale block
  static constexpr int STAGES = 4;
  static constexpr int EPI_WARPS = EPI;     // promotion warps: 8 (2 per TMEM lane quarter) or 16 (4)
  static constexpr int FIRST_EPI = 4;
  static constexpr int THREADS = 32 * (FIRST_EPI + EPI_WARPS);
  static constexpr int COLS_PER_WARP = 256 / (EPI / 4);  // 128 or 64: G columns of each half
  static constexpr int G = COLS_PER_WARP / 2;
  static constexpr int BOXC = G < 64 ? G : 64;             // BF16 store box width
  static constexpr int A_BYTES = BM * BK;                // 16 KB
  static constexpr int B_HALF_BYTES = (HALF / 2) * BK;   // 8 KB: this CTA's 64 rows of one half
  static constexpr int B_BYTES = 2 * B_HALF_BYTES;
  static constexpr int SA_BYTES = BM * 32;               // 4 KB: 128 rows x 8 tf32
  static constexpr int SB_HALF_BYTES = (HALF / 2) * 32;  // 2 KB
  static constexpr int SB_BYTES = 2 * SB_HALF_BYTES;
  static constexpr int STAGE_TX = A_BYTES + B_BYTES + SA_BYTES + SB_BYTES;  // per CTA
  static constexpr int OUT_STAGE_BYTES_PER_WARP = EPI == 16 ? 4096 : 8192;
  // setmaxnreg split of the launch's registers (threads x regs at launch):
  // 8 warps: 384 x 168 >= 128 x 56 + 256 x 224; 16 warps: 640 x 96 = 128 x 32 + 512 x 112.
  static constexpr uint32_t REGS_CONTROL = EPI == 16 ? 32 : 56;
  static constexpr uint32_t REGS_EPILOGUE = EPI == 16 ? 112 : 224;
  static constexpr int TMEM_COLS = 512;
  static constexpr int SMEM_BYTES = STAGES * (A_BYTES + B_BYTES + SA_BYTES + SB_BYTES) +
                                    EPI_WARPS * OUT_STAGE_BYTES_PER_WARP + 512 /*barriers*/ + 1024 /*align*/;
  static_assert(SMEM_BYTES <= 232448, "shared memory");
  static_assert(128 * REGS_CONTROL + 32 * EPI_WARPS * REGS_EPILOGUE <= THREADS * ((65536 / THREADS) & ~7),
                "register split exceeds the launch allocation");
};

// Tile of cluster c (of C) in round r: boustrophedon walk of the tile list.
__device__ __forceinline__ int sp_tile(int round, int c, int C) {
  return round * C + ((round & 1) ? (C - 1 - c) : c);
}

template <int EPI>
__global__ void __launch_bounds__(SpCfg<EPI>::THREADS, 1)
    grouped_wgrad_sp_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                            const __grid_constant__ CUtensorMap tmap_sa, const __grid_constant__ CUtensorMap tmap_sb,
                            const __grid_constant__ CUtensorMap tmap_out, const GemmParams p) {
  using C = SpCfg<EPI>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_a = smem;
  uint8_t* s_b = s_a + C::STAGES * C::A_BYTES;
  uint8_t* s_sa = s_b + C::STAGES * C::B_BYTES;
  uint8_t* s_sb = s_sa + C::STAGES * C::SA_BYTES;
  uint8_t* s_out = s_sb + C::STAGES * C::SB_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_out + C::EPI_WARPS * C::OUT_STAGE_BYTES_PER_WARP);
  uint64_t* full_bar = bars;                    // [STAGES] TMA -> MMA (even CTA's count both CTAs' bytes)
  uint64_t* empty_bar = full_bar + C::STAGES;   // [STAGES] MMA -> TMA (both CTAs)
  uint64_t* tfull_bar = empty_bar + C::STAGES;  // [2] MMA -> promotion, per TMEM slot (both CTAs)
  uint64_t* tempty_bar = tfull_bar + 2;         // [2] promotion of both CTAs -> MMA (even CTA)
  uint64_t* oldout_bar = tempty_bar + 2;        // [EPI_WARPS] previous output -> promotion warp (accumulate)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(oldout_bar + C::EPI_WARPS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cluster = static_cast<int>(cluster_id_x());
  const int nclusters = static_cast<int>(cluster_count_x());
  const int rounds = (p.num_tiles + nclusters - 1) / nclusters;
#if WGRAD_PROFILE
  __shared__ unsigned long long s_prof[kProfSlots];
  __shared__ long long s_issue[8];
  const bool prof_lane = lane == 0 && (warp == 0 || warp == 1 || warp == C::FIRST_EPI);
  if (threadIdx.x < kProfSlots) s_prof[threadIdx.x] = threadIdx.x == kProfCtas ? 1ull : 0ull;
#endif

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::STAGES; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], 2 * C::EPI_WARPS);
    }
    for (int i = 0; i < C::EPI_WARPS; ++i) mbar_init(&oldout_bar[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0 && p.has_operands) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    tma_prefetch_desc(&tmap_sa);
    tma_prefetch_desc(&tmap_sb);
    tma_prefetch_desc(&tmap_out);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
#if WGRAD_PROFILE
  const long long t_cta0 = clock64();
#endif

  if (warp < C::FIRST_EPI) setmaxnreg_dec<C::REGS_CONTROL>();

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
#if WGRAD_PROFILE
      const bool prof_lane = true;
#endif
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint32_t leader_full0 = cluster_addr(&full_bar[0], 0);
      for (int r = 0; r < rounds && ok; ++r) {
        const int tile = sp_tile(r, cluster, nclusters);
        if (tile >= p.num_tiles) continue;
        const TileCoord tc = decode_tile(p, tile, static_cast<int>(rank) * C::BM);
        const int kb0 = __ldg(p.block_offsets + tc.e);
        const int nkb = __ldg(p.block_offsets + tc.e + 1) - kb0;
        const int krow0 = __ldg(p.k_row_offsets + tc.e);
        for (int kb = 0; kb < nkb && ok; ++kb) {
          WGRAD_PROF_T(tw0);
          ok = mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, kDevTimeoutProducer);
          WGRAD_PROF_ADD(kProfProducerWaitStage, tw0);
          if (!ok) break;
#if WGRAD_PROFILE
          s_issue[stage] = clock64();
#endif
          const bool withhold = p.inject == kInjectWithholdFirstLoad && r == 0 && kb == 0;
          const uint32_t lf = leader_full0 + static_cast<uint32_t>(stage * sizeof(uint64_t));
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * C::STAGE_TX);
          if (!withhold) {
            const int kc = krow0 + kb * C::BK;
            const int blk = kb0 + kb;
            uint8_t* b_dst = s_b + stage * C::B_BYTES;
            uint8_t* sb_dst = s_sb + stage * C::SB_BYTES;
            tma_load_2d_pair(s_a + stage * C::A_BYTES, &tmap_a, lf, kc, tc.m0);
            tma_load_2d_pair(b_dst, &tmap_b, lf, kc, tc.n0 + static_cast<int>(rank) * (C::HALF / 2));
            tma_load_2d_pair(b_dst + C::B_HALF_BYTES, &tmap_b, lf, kc,
                             tc.n0 + C::HALF + static_cast<int>(rank) * (C::HALF / 2));
            tma_load_3d_pair(s_sa + stage * C::SA_BYTES, &tmap_sa, lf, 0, tc.m0, blk);
            tma_load_3d_pair(sb_dst, &tmap_sb, lf, 0, tc.n0 + static_cast<int>(rank) * (C::HALF / 2), blk);
            tma_load_3d_pair(sb_dst + C::SB_HALF_BYTES, &tmap_sb, lf, 0,
                             tc.n0 + C::HALF + static_cast<int>(rank) * (C::HALF / 2), blk);
          }
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      // Drain: every stage filled so far has been released by the MMA, so no
      // release arrives after this CTA has exited.
      for (int i = 0; i < C::STAGES && ok; ++i) {
        ok = mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, kDevTimeoutProducer);
        if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
      }
    }
  } else if (warp == 1 && rank == 0) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    constexpr uint32_t idesc_p = umma_idesc_e4m3_f32(2 * C::BM, C::HALF);
    constexpr uint32_t idesc_s = umma_idesc_tf32_f32(2 * C::BM, C::HALF);
    // Descriptors of stage 0; a stage, half or 32-byte K step moves the start
    // address field (bytes >> 4, bits [0, 14)), which never carries out.
    const uint64_t da0 = umma_desc_k_sw128(smem_u32(s_a));
    const uint64_t db0 = umma_desc_k_sw128(smem_u32(s_b));
    const uint64_t dsa0 = umma_desc_k_sw32(smem_u32(s_sa));
    const uint64_t dsb0 = umma_desc_k_sw32(smem_u32(s_sb));
    // shared::cluster addresses of the barriers in CTA 0 and CTA 1
    const uint32_t tfull_c0 = cluster_addr(&tfull_bar[0], 0), tfull_c1 = cluster_addr(&tfull_bar[0], 1);
    const uint32_t empty_c0 = cluster_addr(&empty_bar[0], 0), empty_c1 = cluster_addr(&empty_bar[0], 1);
    int stage = 0, trace_b = 0;
    uint32_t phase = 0, aphase = 0;
    bool ok = true;
    for (int r = 0; r < rounds && ok; ++r) {
      const int tile = sp_tile(r, cluster, nclusters);
      if (tile >= p.num_tiles) continue;
      const TileCoord tc = decode_tile(p, tile);
      const int nkb = __ldg(p.block_offsets + tc.e + 1) - __ldg(p.block_offsets + tc.e);
      // Packed layout: only the 32-row K slices holding the expert's rows in its last block.
      const int klen = __ldg(p.k_row_offsets + tc.e + 1) - __ldg(p.k_row_offsets + tc.e);
      const int last_atoms = min(4, max(1, (klen - (nkb - 1) * C::BK + 31) / 32));
      for (int kb = 0; kb < nkb && ok; ++kb) {
        const int atoms = kb + 1 == nkb ? last_atoms : C::BK / 32;
        const uint64_t da = da0 + static_cast<uint64_t>((stage * C::A_BYTES) >> 4);
        const uint64_t dsa = dsa0 + static_cast<uint64_t>((stage * C::SA_BYTES) >> 4);
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          WGRAD_PROF_T(tm0);
          ok = h == 0 ? mbar_wait2(&tempty_bar[0], aphase ^ 1u, &full_bar[stage], phase, abort_flag, kDevTimeoutMma)
                      : mbar_wait(&tempty_bar[1], aphase ^ 1u, abort_flag, kDevTimeoutMma);
          WGRAD_PROF_ADD(kProfMmaWait, tm0);
#if WGRAD_PROFILE
          if (h == 0 && prof_lane) s_prof[kProfLoadLatency] += static_cast<unsigned long long>(clock64() - s_issue[stage]);
#endif
          WGRAD_PROF_T(tm1);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          WGRAD_TRACE_EV(h == 0 ? kTrMmaReady : kTrMmaHalfReady, trace_b);
          tc_fence_after();
          if (elect_one_sync()) {
            const uint64_t db = db0 + static_cast<uint64_t>((stage * C::B_BYTES + h * C::B_HALF_BYTES) >> 4);
            const uint32_t d_p = tmem_base + static_cast<uint32_t>(h * 2 * C::HALF);
            umma_f8_pair(d_p, da, db, idesc_p, 0u);
            if (atoms > 1) umma_f8_pair(d_p, da + 2, db + 2, idesc_p, 1u);
            if (atoms > 2) umma_f8_pair(d_p, da + 4, db + 4, idesc_p, 1u);
            if (atoms > 3) umma_f8_pair(d_p, da + 6, db + 6, idesc_p, 1u);
            umma_tf32_pair(d_p + C::HALF, dsa, dsb0 + static_cast<uint64_t>((stage * C::SB_BYTES + h * C::SB_HALF_BYTES) >> 4),
                             idesc_s, 0u);
            // the partial is ready in both CTAs; after the second half the stage is free in both
            const uint32_t th = static_cast<uint32_t>(h * sizeof(uint64_t));
            umma_commit_pair(tfull_c0 + th);
            umma_commit_pair(tfull_c1 + th);
            if (h == 1) {
              const uint32_t es = static_cast<uint32_t>(stage * sizeof(uint64_t));
              umma_commit_pair(empty_c0 + es);
              umma_commit_pair(empty_c1 + es);
            }
          }
          __syncwarp();
          WGRAD_TRACE_EV(h == 0 ? kTrMmaIssued : kTrMmaHalfIssued, trace_b);
          WGRAD_PROF_ADD(kProfMmaIssue, tm1);
        }
        if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        aphase ^= 1u;
        ++trace_b;
      }
    }
  } else if (warp >= C::FIRST_EPI) {
    // ------------------------------------------------------------ promotion + epilogue (both CTAs)
    setmaxnreg_inc<C::REGS_EPILOGUE>();
    const int ew = warp - C::FIRST_EPI;  // 0 .. EPI_WARPS - 1
    const int quarter = warp & 3;        // TMEM lane quarter this warp may access
    const int cg = ew >> 2;              // G-column group within each half
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    uint8_t* stage_out = s_out + ew * C::OUT_STAGE_BYTES_PER_WARP;
    const uint32_t tempty_leader0 = cluster_addr(&tempty_bar[0], 0);
    uint32_t aphase = 0, oldout_phase = 0;
    int trace_b = 0;
    bool ok = true;
#if WGRAD_DEBUG_MODES
    const bool unit_scales = p.mode == kModeUnscaled;  // raw FP8 product only
    const bool unit_raw = p.mode == kModeScaleOnly;    // scale product only
#endif
    for (int r = 0; r < rounds && ok; ++r) {
      const int tile = sp_tile(r, cluster, nclusters);
      if (tile >= p.num_tiles) continue;
      const TileCoord tc = decode_tile(p, tile, static_cast<int>(rank) * C::BM);
      const int nkb = __ldg(p.block_offsets + tc.e + 1) - __ldg(p.block_offsets + tc.e);
      float fin[C::COLS_PER_WARP];
#pragma unroll
      for (int j = 0; j < C::COLS_PER_WARP; ++j) fin[j] = 0.f;

      for (int kb = 0; kb < nkb && ok; ++kb) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (ew == 0 && h == 0) WGRAD_TRACE_EV(kTrEpiWaitStart, trace_b);
          WGRAD_PROF_T(te0);
          ok = mbar_wait(&tfull_bar[h], aphase, abort_flag, kDevTimeoutEpilogue);
          WGRAD_PROF_ADD(kProfEpiWait, te0);
          WGRAD_PROF_T(te1);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) continue;
          if (ew == 0 && h == 0) WGRAD_TRACE_EV(kTrEpiReady, trace_b);
          tc_fence_after();
          const uint32_t t_p = tmem_base + lane_addr + static_cast<uint32_t>(h * 2 * C::HALF + cg * C::G);
          // SP_CHUNK-column pieces of P and S; the slot goes back to the MMA
          // thread as soon as the last piece is in registers.
          uint32_t rp[SP_CHUNK], rs[SP_CHUNK];
#pragma unroll
          for (int c = 0; c < C::G / SP_CHUNK; ++c) {
            tmem_ld_chunk(t_p + c * SP_CHUNK, rp);
            tmem_ld_chunk(t_p + C::HALF + c * SP_CHUNK, rs);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < SP_CHUNK; ++i) asm volatile("" : "+r"(rp[i]), "+r"(rs[i]));
            if (c == C::G / SP_CHUNK - 1) {
              tc_fence_before();
              __syncwarp();
              if (elect_one_sync()) {
                if (rank != 0) mbar_arrive_cluster(tempty_leader0 + static_cast<uint32_t>(h * sizeof(uint64_t)));
                else mbar_arrive(&tempty_bar[h]);
              }
              if (ew == 0) WGRAD_TRACE_EV(h == 0 ? kTrEpiReleased : kTrEpiDone, trace_b);
            }
            float* f = &fin[h * C::G + c * SP_CHUNK];
#pragma unroll
            for (int j = 0; j < SP_CHUNK; j += 2) {
#if WGRAD_DEBUG_MODES
              const float p0 = unit_raw ? 1.f : __uint_as_float(rp[j]);
              const float p1 = unit_raw ? 1.f : __uint_as_float(rp[j + 1]);
              const float s0 = unit_scales ? 1.f : __uint_as_float(rs[j]);
              const float s1 = unit_scales ? 1.f : __uint_as_float(rs[j + 1]);
              fma_f32x2(f[j], f[j + 1], p0, p1, s0, s1, f[j], f[j + 1]);
#else
              fma_f32x2(f[j], f[j + 1], __uint_as_float(rp[j]), __uint_as_float(rp[j + 1]), __uint_as_float(rs[j]),
                        __uint_as_float(rs[j + 1]), f[j], f[j + 1]);
#endif
            }
          }
          WGRAD_PROF_ADD(kProfEpiPromote, te1);
        }
        WGRAD_PROF_INC(kProfKBlocks);
        aphase ^= 1u;
        ++trace_b;
      }
      if (!ok) break;

      // -------------------------------------------------------- epilogue store
      WGRAD_PROF_T(ts0);
      WGRAD_PROF_INC(kProfTiles);
      const int col0 = tc.n0 + cg * C::G;
#if WGRAD_DEBUG_MODES
      if (p.mode == kModeCoordM || p.mode == kModeCoordN || p.mode == kModeScaleOnly) {
        const int g_row = tc.m0 + quarter * 32 + lane;
#pragma unroll
        for (int j = 0; j < C::COLS_PER_WARP; ++j) {
          fin[j] = p.mode == kModeCoordM ? static_cast<float>(g_row)
                 : p.mode == kModeCoordN ? static_cast<float>(col0 + (j / C::G) * C::HALF + (j % C::G))
                                         : fin[j] * 1048576.0f;  // 2^20, as the reference
        }
      }
#endif
      WGRAD_PROF_T(ts1);
      if (lane == 0) bulk_wait_group_read0();
      __syncwarp();
      WGRAD_PROF_ADD(kProfEpiStoreWait, ts1);
      ok = store_warp_tile<C::COLS_PER_WARP, C::OUT_STAGE_BYTES_PER_WARP, C::HALF, C::G, C::BOXC>(
          fin, tmap_out, p, tc, quarter, lane, col0, stage_out, &oldout_bar[ew], oldout_phase, abort_flag);
      if (!ok) break;
      WGRAD_PROF_ADD(kProfEpiStore, ts0);
    }
    if (lane == 0) bulk_wait_group0();  // all output writes complete before exit
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no cross-CTA arrival or UMMA is left in flight
#if WGRAD_PROFILE
  if (threadIdx.x < kProfSlots)
    atomicAdd(&g_wgrad_prof[threadIdx.x], threadIdx.x == kProfCtaCycles
                                              ? static_cast<unsigned long long>(clock64() - t_cta0)
                                              : s_prof[threadIdx.x]);
#endif
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

// Split fp32 scales into TF32 operand rows of the scale-product UMMA:
//   lhs scale s -> [hi, hi, lo, lo],  rhs scale s -> [hi, lo, hi, lo]
// (hi = s truncated to TF32, lo = (s - hi) truncated to TF32; s - hi is exact).
// Only the scale blocks of the launched expert range [block_offsets[0],
// block_offsets[E]) are converted (the range is read on the device).
__global__ void __launch_bounds__(256) scale_operand_kernel(const float* __restrict__ sa, const float* __restrict__ sb,
                                                            float4* __restrict__ opa, float4* __restrict__ opb,
                                                            int64_t m, int64_t n, const int32_t* block_offsets,
                                                            int num_experts, int64_t total_blocks) {
  int64_t b0 = __ldg(block_offsets);
  int64_t b1 = __ldg(block_offsets + num_experts);
  b0 = b0 < 0 ? 0 : (b0 > total_blocks ? total_blocks : b0);
  b1 = b1 < b0 ? b0 : (b1 > total_blocks ? total_blocks : b1);
  const int64_t na = (b1 - b0) * m, nb = (b1 - b0) * n;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  auto split = [](float s, float& hi, float& lo) {
    hi = __uint_as_float(__float_as_uint(s) & 0xFFFFE000u);
    lo = __uint_as_float(__float_as_uint(s - hi) & 0xFFFFE000u);
  };
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < na + nb; i += stride) {
    float hi, lo;
    if (i < na) {
      const int64_t idx = b0 * m + i;
      split(__ldg(sa + idx), hi, lo);
      opa[idx] = make_float4(hi, hi, lo, lo);
    } else {
      const int64_t idx = b0 * n + (i - na);
      split(__ldg(sb + idx), hi, lo);
      opb[idx] = make_float4(hi, lo, hi, lo);
    }
  }
}

}  // namespace

cudaError_t launch_scale_operands(const float* sa, const float* sb, void* opa, void* opb, int64_t m, int64_t n,
                                  const int32_t* block_offsets, int num_experts, int64_t total_blocks, int sm_count,
                                  cudaStream_t stream) {
  const int grid = sm_count * 8;
  scale_operand_kernel<<<grid, 256, 0, stream>>>(sa, sb, static_cast<float4*>(opa), static_cast<float4*>(opb), m, n,
                                                 block_offsets, num_experts, total_blocks);
  return cudaGetLastError();
}

template <int EPI>
static cudaError_t launch_sp(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tsa,
                             const CUtensorMap& tsb, const CUtensorMap& to, const GemmParams& p, int grid,
                             cudaStream_t stream) {
  using C = SpCfg<EPI>;
  const cudaError_t err = configure_once<grouped_wgrad_sp_kernel<EPI>>(C::SMEM_BYTES);
  if (err != cudaSuccess) return err;
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
  return cudaLaunchKernelEx(&cfg, grouped_wgrad_sp_kernel<EPI>, ta, tb, tsa, tsb, to, p);
}

cudaError_t launch_grouped_wgrad_sp(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tsa,
                                    const CUtensorMap& tsb, const CUtensorMap& to, const GemmParams& p, int grid,
                                    cudaStream_t stream) {
  return p.epi_warps == 16 ? launch_sp<16>(ta, tb, tsa, tsb, to, p, grid, stream)
                           : launch_sp<8>(ta, tb, tsa, tsb, to, p, grid, stream);
}

}  // namespace wgrad
