// UMMA issue-rate probe: one thread per SM issues back-to-back tcgen05.mma
// (128 x N x 128 per K block, four K=32 UMMAs) on operand tiles that stay in
// shared memory, optionally while a second warp streams 1-D bulk copies from
// L2 into a separate shared-memory ring and a third chases a dependent chain of
// ld.shared. Prints SM cycles per K block, the aggregate FP8 rate, the
// bulk-copy bytes per SM cycle and the latency of one ld.shared under that load.
//
// It separates candidate bounds of the grouped Wgrad kernels: the tensor pipe
// itself, tensor-core reads of shared memory competing with TMA writes into
// it, the latency of the operand loads (bytes in flight), and the latency the
// promotion and scale-factor warps see on their shared-memory loads.
//
// Build: python sm90-fp8-wgrad_b200/build_ext.py --probes
// Run:   sm90-fp8-wgrad_b200/sm90_fp8_wgrad/_lib/umma_rate
#include <cstdint>
#include <cstdio>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../csrc/ptx.cuh"

using namespace wgrad;

namespace {

constexpr int kRing = 4;  // bulk-copy ring slots

template <int N, bool MX, bool CP_EACH = false, bool RANDOM = false>
__global__ void __launch_bounds__(128, 1)
    umma_rate_kernel(int iters, unsigned long long* out, const uint8_t* src, int ring_kb, int mma_on) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_a = smem;                  // 128 rows x 128 B
  uint8_t* s_b = smem + 16384;          // N rows x 128 B
  uint8_t* s_sf = smem + (RANDOM ? 4 : 1) * (16384 + N * 128);  // scale factors, 512 + 1024 B
  uint8_t* ring = s_sf + 2048;          // bulk-copy ring
  __shared__ uint64_t done_bar, ring_bar[kRing];
  __shared__ uint32_t holder;
  __shared__ int abort_flag;
  __shared__ volatile int mma_done;
  __shared__ uint32_t chase[256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // e4m3 1.0 operands (RANDOM: four stages of pseudo-random finite e4m3 bytes,
  // rotated per K block as the kernels' operand ring); E8M0 1.0 scale factors
  constexpr int STAGE_BYTES = 16384 + N * 128;
  for (int i = threadIdx.x; i < (RANDOM ? 4 : 1) * STAGE_BYTES / 4; i += blockDim.x) {
    uint32_t w = 0x38383838u;
    if (RANDOM) {
      uint32_t h = static_cast<uint32_t>(i) * 2654435761u + blockIdx.x * 40503u;
      h ^= h >> 13;
      h *= 0x5bd1e995u;
      h ^= h >> 15;
      w = h & 0x77777777u;  // clear bit 7 and bit 3 of each byte: finite, |x| < 448
    }
    reinterpret_cast<uint32_t*>(smem)[i] = w;
  }
  for (int i = threadIdx.x; i < 2048 / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(s_sf)[i] = 0x7F7F7F7Fu;
  if (threadIdx.x == 0) {
    mbar_init(&done_bar, 1);
    for (int i = 0; i < kRing; ++i) mbar_init(&ring_bar[i], 1);
    abort_flag = 0;
    mma_done = 0;
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < 256; i += blockDim.x) chase[i] = static_cast<uint32_t>((i * 37 + 11) & 255);
  if (warp == 1) {
    tmem_alloc(&holder, 512);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = holder;
  volatile int* abort_p = &abort_flag;

  if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = MX ? umma_idesc_mxf8_e4m3_ue8m0(128, N) : umma_idesc_e4m3_f32(128, N);
    const uint32_t a = smem_u32(s_a), b = smem_u32(s_b);
    const uint32_t sf = tmem + 384;  // scale factors behind a 256-column accumulator
    if (MX) {
      tmem_cp_32x128b_warpx4(sf, smem_desc_rows16(smem_u32(s_sf)));
      tmem_cp_32x128b_warpx4(sf + 4, smem_desc_rows16(smem_u32(s_sf) + 512));
      tmem_cp_32x128b_warpx4(sf + 8, smem_desc_rows16(smem_u32(s_sf) + 1024));
    }
    const long long t0 = clock64();
    for (int it = 0; it < iters * mma_on; ++it) {
      // CP_EACH: fresh scale factors for every K block, into one of 4 rotating
      // 16-column TMEM stages, as the UE8M0 kernel copies them
      const uint32_t sfs = CP_EACH ? sf + static_cast<uint32_t>((it & 3) * 16) : sf;
      if (CP_EACH) {
        tmem_cp_32x128b_warpx4(sfs, smem_desc_rows16(smem_u32(s_sf)));
        tmem_cp_32x128b_warpx4(sfs + 4, smem_desc_rows16(smem_u32(s_sf) + 512));
        tmem_cp_32x128b_warpx4(sfs + 8, smem_desc_rows16(smem_u32(s_sf) + 1024));
      }
      const uint32_t st = RANDOM ? static_cast<uint32_t>((it & 3) * (16384 + N * 128)) : 0u;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint64_t da = umma_desc_k_sw128(a + st + k * 32), db = umma_desc_k_sw128(b + st + k * 32);
        if (MX) umma_mxf8(tmem, da, db, idesc, sfs, sfs + 4, 1u);
        else umma_f8(tmem, da, db, idesc, 1u);
      }
    }
    umma_commit(&done_bar);
    const bool ok = mbar_wait(&done_bar, 0, abort_p, kDevTimeoutMma);
    const long long t1 = clock64();
    mma_done = 1;
    if (blockIdx.x == 0) {
      out[0] = static_cast<unsigned long long>(t1 - t0);
      out[1] = ok ? 1ull : 0ull;
    }
  }
  if (warp == 2 && lane == 0) {
    // dependent ld.shared chain while the UMMAs (and bulk copies) run
    uint32_t idx = 0;
    unsigned long long loads = 0;
    const long long t0 = clock64();
    while ((!mma_done || loads == 0) && loads < 50000000ull) {
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(idx) : "r"(smem_u32(&chase[idx & 255])) : "memory");
      }
      loads += 64;
      if (!mma_on && loads >= 4096) break;
    }
    const long long t1 = clock64();
    if (blockIdx.x == 0) {
      out[4] = loads;
      out[5] = static_cast<unsigned long long>(t1 - t0);
      out[6] = idx;
    }
  }
  if (warp == 3 && lane == 0 && ring_kb > 0) {
    const uint32_t chunk = static_cast<uint32_t>(ring_kb) * 1024u / kRing;
    const uint8_t* base = src + static_cast<size_t>(blockIdx.x) * 65536;  // 64 KB per CTA, L2-resident
    uint32_t phase[kRing] = {0, 0, 0, 0};
    unsigned long long bytes = 0, it = 0;
    const long long t0 = clock64();
    for (int s = 0; s < kRing; ++s) {
      mbar_arrive_expect_tx(&ring_bar[s], chunk);
      bulk_load_1d(ring + s * chunk, base + s * chunk % 65536, chunk, &ring_bar[s]);
    }
    bool ok = true;
    while (!mma_done && ok && it < 100000000ull) {
      const int s = static_cast<int>(it % kRing);
      ok = mbar_wait(&ring_bar[s], phase[s], abort_p, kDevTimeoutProducer);
      if (!ok) break;
      phase[s] ^= 1u;
      bytes += chunk;
      ++it;
      mbar_arrive_expect_tx(&ring_bar[s], chunk);
      bulk_load_1d(ring + s * chunk, base + (it * chunk) % 65536, chunk, &ring_bar[s]);
    }
    for (int s = 0; s < kRing; ++s) (void)mbar_wait(&ring_bar[s], phase[s], abort_p, kDevTimeoutProducer);
    const long long t1 = clock64();
    if (blockIdx.x == 0) {
      out[2] = bytes;
      out[3] = static_cast<unsigned long long>(t1 - t0);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int N, bool MX, bool CP_EACH = false, bool RANDOM = false>
int run(const char* name, int sms, int ring_kb, const uint8_t* src, unsigned long long* d_out, int mma_on = 1) {
  const int iters = 4096;
  const int smem = 1024 + (RANDOM ? 4 : 1) * (16384 + N * 128) + 2048 + ring_kb * 1024;
  if (cudaFuncSetAttribute(umma_rate_kernel<N, MX, CP_EACH, RANDOM>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return 1;
  for (int rep = 0; rep < 2; ++rep) {
    cudaMemset(d_out, 0, 8 * sizeof(unsigned long long));
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0);
    umma_rate_kernel<N, MX, CP_EACH, RANDOM><<<sms, 128, smem>>>(iters, d_out, src, ring_kb, mma_on);
    cudaEventRecord(e1);
    const cudaError_t err = cudaEventSynchronize(e1);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    unsigned long long h[7] = {0, 0, 0, 0, 0, 0, 0};
    cudaMemcpy(h, d_out, sizeof(h), cudaMemcpyDeviceToHost);
    const double flops = 2.0 * 128 * N * 128 * static_cast<double>(iters) * sms;
    std::printf("%-18s SMs %3d  UMMA %s bulk ring %3d KB: %6.1f cycles / K block (tensor-pipe floor %d), "
                "%5.0f TFLOP/s, bulk %5.1f B/cycle/SM, ld.shared %6.1f cycles, wait ok %llu, %s\n",
                name, sms, mma_on ? "on " : "off", ring_kb, mma_on ? static_cast<double>(h[0]) / iters : 0.0, 2 * N,
                mma_on ? flops / (ms * 1e-3) / 1e12 : 0.0,
                h[3] ? static_cast<double>(h[2]) / static_cast<double>(h[3]) : 0.0,
                h[4] ? static_cast<double>(h[5]) / static_cast<double>(h[4]) : 0.0, h[1], cudaGetErrorString(err));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (err != cudaSuccess) return 1;
  }
  return 0;
}

// TMEM read throughput: each of 4 * W warps (W per lane quarter) loads
// 32 lanes x 32 columns (4 KB) per tcgen05.ld, `inflight` loads before each
// wait, `reps` times; prints bytes per SM cycle.
template <int INFLIGHT>
__global__ void __launch_bounds__(512, 1) tmem_ld_rate_kernel(int reps, unsigned long long* out) {
  __shared__ uint32_t holder;
  const int warp = threadIdx.x >> 5;
  if (warp == 0) {
    tmem_alloc(&holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = holder + (static_cast<uint32_t>((warp & 3) * 32) << 16);
  const uint32_t col0 = static_cast<uint32_t>((warp >> 2) * 32 * INFLIGHT) & 511u;
  uint32_t acc = 0;
  const long long t0 = clock64();
  for (int r = 0; r < reps; ++r) {
    uint32_t v[INFLIGHT][32];
#pragma unroll
    for (int i = 0; i < INFLIGHT; ++i) tmem_ld_32x32b_x32(tmem + ((col0 + 32u * i) & 511u), v[i]);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < INFLIGHT; ++i) acc ^= v[i][0] ^ v[i][31];
  }
  const long long t1 = clock64();
  __syncthreads();
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    out[0] = static_cast<unsigned long long>(t1 - t0);
    out[1] = acc;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(holder, 512);
  }
}

template <int INFLIGHT>
int run_tmem(int sms, int warps, unsigned long long* d_out) {
  const int reps = 4096;
  cudaMemset(d_out, 0, 2 * sizeof(unsigned long long));
  tmem_ld_rate_kernel<INFLIGHT><<<sms, 32 * warps>>>(reps, d_out);
  const cudaError_t err = cudaDeviceSynchronize();
  unsigned long long h[2] = {0, 0};
  cudaMemcpy(h, d_out, sizeof(h), cudaMemcpyDeviceToHost);
  const double bytes = 4096.0 * INFLIGHT * reps * warps;  // per SM
  std::printf("tcgen05.ld 32x32b.x32, %2d warps, %d in flight: %6.1f B/cycle/SM (%.1f cycles per 4 KB load), %s\n",
              warps, INFLIGHT, h[0] ? bytes / static_cast<double>(h[0]) : 0.0,
              h[0] ? static_cast<double>(h[0]) * warps / (static_cast<double>(reps) * INFLIGHT * warps) : 0.0,
              cudaGetErrorString(err));
  return err == cudaSuccess ? 0 : 1;
}

}  // namespace

int main() {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  uint8_t* src = nullptr;
  unsigned long long* d_out = nullptr;
  if (cudaMalloc(&src, static_cast<size_t>(sms + 1) * 65536) != cudaSuccess) return 1;
  cudaMemset(src, 0, static_cast<size_t>(sms + 1) * 65536);
  cudaMalloc(&d_out, 8 * sizeof(unsigned long long));
  int rc = 0;
  rc |= run<256, false>("f8f6f4 N=256", sms, 0, src, d_out, 0);
  rc |= run<256, false>("f8f6f4 N=256", sms, 128, src, d_out, 0);
  rc |= run<256, false>("f8f6f4 N=256", 1, 0, src, d_out);
  rc |= run<256, false>("f8f6f4 N=256", sms, 0, src, d_out);
  rc |= run<256, false>("f8f6f4 N=256", sms, 64, src, d_out);
  rc |= run<256, false>("f8f6f4 N=256", sms, 128, src, d_out);
  rc |= run<128, false>("f8f6f4 N=128", sms, 0, src, d_out);
  rc |= run<192, true>("mxf8f6f4 N=192", sms, 0, src, d_out);
  rc |= run<192, true>("mxf8f6f4 N=192", sms, 64, src, d_out);
  rc |= run<192, true, true>("mxf8 N=192 +cp/blk", sms, 0, src, d_out);
  rc |= run<192, true, true, true>("mxf8 N=192 rand4", sms, 0, src, d_out);
  rc |= run<256, false, false, true>("f8f6f4 N=256 rand4", sms, 0, src, d_out);
  rc |= run_tmem<1>(sms, 4, d_out);
  rc |= run_tmem<2>(sms, 4, d_out);
  rc |= run_tmem<1>(sms, 8, d_out);
  rc |= run_tmem<2>(sms, 8, d_out);
  rc |= run_tmem<2>(sms, 16, d_out);
  cudaFree(src);
  cudaFree(d_out);
  return rc;
}
