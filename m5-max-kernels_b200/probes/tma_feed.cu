// TMA feed probe: how fast one SM's shared memory fills from L2 / HBM.
//
// The GEMM's CTAs stream 128-byte k-slices of A and W into a shared-memory
// ring with tiled TMA loads.  This load-only kernel (no MMAs) issues the same
// kind of copies from one thread per CTA, one CTA per SM, and reports the
// bytes landed per SM per second for:
//   * copy shapes: 2D boxes of 128 rows x 128 bytes (the GEMM's), 256-row 2D
//     boxes, 3D boxes of 128 or 256 rows x two k-blocks, with 32 or 64 KB
//     ring stages and 2-6 stages in flight;
//   * 8, 74 and 148 active SMs, with the operands resident in L2 or not;
//   * a CTA pair in which one CTA forwards half of each stage to the other
//     through distributed shared memory (cp.async.bulk shared::cta ->
//     shared::cluster; no multicast), and that forwarding alone.
// Every wait is bounded (300 ms); a timed-out wait sets a status bit, and the
// program stops at the first configuration that reports one.
//
// Build and run (one GPU):
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 \
//        -I m5-max-kernels_b200/csrc -I include m5-max-kernels_b200/probes/tma_feed.cu \
//        -o tma_feed && ./tma_feed
#include "common.cuh"
#include <cudaTypedefs.h>
#include <cstdio>
#include <cstdlib>
#include <vector>
#include <algorithm>
using namespace m5b;

constexpr int STAGE = 32768;
constexpr int HALF = 16384;
constexpr int L0 = 2;  // forward lag on rank 0

struct Params {
  CUtensorMap mapA, mapB, mapA2, map3a, map3b, map3c;
  int stage_bytes;
  const uint8_t* gA; const uint8_t* gB;
  int mblocks, nblocks, nk, iters, mode;
  unsigned int* status;
  unsigned long long* times;
};

__device__ __forceinline__ bool wait_b(uint64_t* bar, uint32_t parity, unsigned int* status,
                                       unsigned code, bool& dead) {
  if (dead) return false;
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > 300000000ull) {
      atomicOr(status, code);
      dead = true;
      return false;
    }
  }
  return true;
}
// drain wait: bounded, ignores the dead flag
__device__ __forceinline__ void wait_drain(uint64_t* bar, uint32_t parity, unsigned int* status) {
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > 300000000ull) { atomicOr(status, 0x100u); return; }
  }
}

template <int S>
__global__ void __launch_bounds__(32, 1) probe(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[S];
  __shared__ __align__(8) uint64_t pempty[S];
  const int mode = p.mode;
  const bool clustered = mode == 1 || mode == 2 || mode == 3;
  const uint32_t rank = clustered ? cluster_rank() : 0;
  const int cid = clustered ? blockIdx.x / 2 : blockIdx.x;
  const int mb = cid % p.mblocks;
  const int nb = clustered ? (2 * cid + (int)rank) % p.nblocks : (cid / p.mblocks) % p.nblocks;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(&full[s], 1); mbar_init(&pempty[s], 1); }
    fence_mbarrier_init();
  }
  __syncwarp();
  if (clustered) cluster_sync();
  const unsigned long long t0 = globaltimer_ns();
  bool dead = false;
  if (threadIdx.x == 0) {
    const int iters = p.iters;
    if (mode == 0 || mode == 3 || mode == 4 || mode >= 6) {
      // every CTA loads both boxes itself (mode 3: same, launched in clusters of 2)
      for (int it = 0; it < iters; ++it) {
        const int s = it % S; const uint32_t u = it / S;
        if (u >= 1 && !wait_b(&full[s], (u - 1) & 1, p.status, 1u, dead)) break;
        const int kb = it % p.nk;
        mbar_arrive_expect_tx(&full[s], p.stage_bytes);
        uint8_t* st = ring + s * p.stage_bytes;
        if (mode == 7) {          // one 3D box: 128 rows x 2 k-blocks (32 KB)
          tma_load_3d(st, &p.map3a, &full[s], 0, mb * 128, (2 * kb) % p.nk);
        } else if (mode == 8) {   // two 3D boxes of 128 rows x 2 k-blocks (64 KB)
          tma_load_3d(st, &p.map3a, &full[s], 0, mb * 128, (2 * kb) % p.nk);
          tma_load_3d(st + 32768, &p.map3b, &full[s], 0, nb * 128, (2 * kb) % p.nk);
        } else if (mode == 9) {   // one 3D box: 256 rows x 2 k-blocks (64 KB)
          tma_load_3d(st, &p.map3c, &full[s], 0, (mb & ~1) * 128, (2 * kb) % p.nk);
        } else if (mode == 10) {  // four 2D boxes: A and B, two k-blocks each (64 KB)
          for (int q = 0; q < 2; ++q) {
            tma_load_2d(st + q * 16384, &p.mapA, &full[s], ((2 * kb + q) % p.nk) * 128, mb * 128);
            tma_load_2d(st + 32768 + q * 16384, &p.mapB, &full[s], ((2 * kb + q) % p.nk) * 128, nb * 128);
          }
        } else if (mode == 4) {
          const uint8_t* a = p.gA + (size_t(mb) * p.nk + kb) * HALF;
          const uint8_t* b = p.gB + (size_t(nb) * p.nk + kb) * HALF;
          bulk_load_g2s(st, a, HALF, &full[s]);
          bulk_load_g2s(st + HALF, b, HALF, &full[s]);
        } else if (mode == 6) {
          tma_load_2d(st, &p.mapA2, &full[s], kb * 128, (mb & ~1) * 128);
        } else {
          tma_load_2d(st, &p.mapA, &full[s], kb * 128, mb * 128);
          tma_load_2d(st + HALF, &p.mapB, &full[s], kb * 128, nb * 128);
        }
      }
      for (int s = 0; s < S; ++s) {
        const int uses = (iters - s + S - 1) / S;
        if (uses >= 1) wait_drain(&full[s], (uses - 1) & 1, p.status);
      }
    } else if (rank == 0) {
      const bool load = mode == 1;
      const uint32_t peer_ring = map_to_rank(ring, 1);
      const uint32_t peer_full = map_to_rank(&full[0], 1);
      for (int j = 0; j < iters + L0 && !dead; ++j) {
        const int f = j - L0;
        if (f >= 0 && f < iters) {
          const int sf = f % S; const uint32_t uf = f / S;
          if (load && !wait_b(&full[sf], uf & 1, p.status, 2u, dead)) break;
          if (uf >= 1 && !wait_b(&pempty[sf], (uf - 1) & 1, p.status, 4u, dead)) break;
          bulk_copy_s2cluster(peer_ring + sf * STAGE, ring + sf * STAGE, HALF, peer_full + sf * 8);
          bulk_commit_group();
        }
        if (j < iters) {
          const int s = j % S; const uint32_t u = j / S;
          if (load) {
            if (u >= 1) asm volatile("cp.async.bulk.wait_group.read 4;" ::: "memory");  // S - L0
            const int kb = j % p.nk;
            mbar_arrive_expect_tx(&full[s], STAGE);
            tma_load_2d(ring + s * STAGE, &p.mapA, &full[s], kb * 128, mb * 128);
            tma_load_2d(ring + s * STAGE + HALF, &p.mapB, &full[s], kb * 128, nb * 128);
          } else {
            asm volatile("cp.async.bulk.wait_group.read 4;" ::: "memory");
          }
        }
      }
      bulk_wait_group0();
      if (load)
        for (int s = 0; s < S; ++s) {
          const int uses = (iters - s + S - 1) / S;
          if (uses >= 1) wait_drain(&full[s], (uses - 1) & 1, p.status);
        }
    } else {
      const bool load = mode == 1;
      const uint32_t peer_pempty = map_to_rank(&pempty[0], 0);
      for (int j = 0; j < iters + S - 1 && !dead; ++j) {
        if (j < iters) {
          const int s = j % S;
          mbar_arrive_expect_tx(&full[s], load ? STAGE : HALF);
          if (load) {
            const int kb = j % p.nk;
            tma_load_2d(ring + s * STAGE + HALF, &p.mapB, &full[s], kb * 128, nb * 128);
          }
        }
        const int c = j - (S - 1);
        if (c >= 0) {
          const int sc = c % S; const uint32_t uc = c / S;
          if (!wait_b(&full[sc], uc & 1, p.status, 8u, dead)) break;
          mbar_arrive_cluster(peer_pempty + sc * 8);
        }
      }
      for (int s = 0; s < S; ++s) {
        const int uses = (iters - s + S - 1) / S;
        if (uses >= 1) wait_drain(&full[s], (uses - 1) & 1, p.status);
      }
    }
  }
  __syncwarp();
  const unsigned long long t1 = globaltimer_ns();
  if (threadIdx.x == 0) { p.times[2 * blockIdx.x] = t0; p.times[2 * blockIdx.x + 1] = t1; }
  if (clustered) cluster_sync();
}

static PFN_cuTensorMapEncodeTiled_v12000 g_enc;
static void mkmap(CUtensorMap* m, void* ptr, int rows, int k, int boxrows = 128) {
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)k};
  cuuint32_t box[2] = {128, (cuuint32_t)boxrows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, ptr, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) { printf("encode failed %d\n", r); exit(1); }
}
static void mkmap3(CUtensorMap* m, void* ptr, int rows, int k, int boxrows, int boxkb) {
  cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)(k / 128)};
  cuuint64_t strides[2] = {(cuuint64_t)k, 128};
  cuuint32_t box[3] = {128, (cuuint32_t)boxrows, (cuuint32_t)boxkb};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, ptr, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) { printf("encode3 failed %d\n", r); exit(1); }
}
#define CK(x) do { cudaError_t e_ = (x); if (e_ != cudaSuccess) { printf("CUDA %s at %d\n", cudaGetErrorString(e_), __LINE__); exit(1);} } while (0)

int main() {
  void* fn = nullptr; cudaDriverEntryPointQueryResult q;
  CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
  g_enc = (PFN_cuTensorMapEncodeTiled_v12000)fn;
  const int K = 16384;
  struct Shape { int arows, brows; const char* name; };
  Shape shapes[2] = {{512, 2048, "L2-resident (A 8 MB + B 32 MB)"}, {4096, 4096, "DRAM (A 64 MB + B 64 MB)"}};
  uint8_t *dA, *dB;
  CK(cudaMalloc(&dA, size_t(4096) * K)); CK(cudaMalloc(&dB, size_t(4096) * K));
  CK(cudaMemset(dA, 1, size_t(4096) * K)); CK(cudaMemset(dB, 2, size_t(4096) * K));
  unsigned int* status; unsigned long long* times;
  CK(cudaMalloc(&status, 4)); CK(cudaMemset(status, 0, 4));
  CK(cudaMalloc(&times, 2 * 148 * 8));
  const int smem = 200 * 1024;
  CK(cudaFuncSetAttribute(probe<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  CK(cudaFuncSetAttribute(probe<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  CK(cudaFuncSetAttribute(probe<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  CK(cudaFuncSetAttribute(probe<6>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));

  cudaEvent_t e0, e1; CK(cudaEventCreate(&e0)); CK(cudaEventCreate(&e1));
  const int grids[] = {8, 74, 148};  // active SMs (CTAs)
  for (int sh = 0; sh < 2; ++sh) {
    Params p{};
    mkmap(&p.mapA, dA, shapes[sh].arows, K);
    mkmap(&p.mapB, dB, shapes[sh].brows, K);
    mkmap(&p.mapA2, dA, shapes[sh].arows, K, 256);
    mkmap3(&p.map3a, dA, shapes[sh].arows, K, 128, 2);
    mkmap3(&p.map3b, dB, shapes[sh].brows, K, 128, 2);
    mkmap3(&p.map3c, dA, shapes[sh].arows, K, 256, 2);
    p.gA = dA; p.gB = dB;
    p.mblocks = shapes[sh].arows / 128; p.nblocks = shapes[sh].brows / 128; p.nk = K / 128;
    p.status = status; p.times = times;
    printf("== %s\n", shapes[sh].name);
    // copy shapes (r: rows per box, kb: k-blocks per box) and stage sizes
    const int modes[] = {0, 4, 6, 7, 8, 9, 10};
    const int sbytes[] = {32768, 32768, 32768, 32768, 65536, 65536, 65536};
    const char* mname[] = {"2D 2x(128r x 1kb) 32K", "bulk 2x16KB contiguous", "2D 1x(256r x 1kb) 32K",
                           "3D 1x(128r x 2kb) 32K", "3D 2x(128r x 2kb) 64K", "3D 1x(256r x 2kb) 64K",
                           "2D 4x(128r x 1kb) 64K"};
    for (int mi = 0; mi < 7; ++mi) {
      const int mode = modes[mi];
      p.stage_bytes = sbytes[mi];
      for (int sdepth : {2, 3, 4, 6}) {
        if (sdepth * sbytes[mi] > 196608) continue;
        for (int g : grids) {
          p.mode = mode; p.iters = 6144;
          cudaLaunchConfig_t cfg{}; cfg.gridDim = dim3(g); cfg.blockDim = dim3(32);
          cfg.dynamicSmemBytes = 200 * 1024; cfg.stream = 0;
          cfg.attrs = nullptr; cfg.numAttrs = 0;
          float ms = 0;
          for (int rep = 0; rep < 2; ++rep) {
            CK(cudaEventRecord(e0));
            if (sdepth == 2) CK(cudaLaunchKernelEx(&cfg, probe<2>, p));
            if (sdepth == 3) CK(cudaLaunchKernelEx(&cfg, probe<3>, p));
            if (sdepth == 4) CK(cudaLaunchKernelEx(&cfg, probe<4>, p));
            if (sdepth == 6) CK(cudaLaunchKernelEx(&cfg, probe<6>, p));
            CK(cudaEventRecord(e1));
            CK(cudaEventSynchronize(e1));
          }
          CK(cudaEventElapsedTime(&ms, e0, e1));
          unsigned int st; CK(cudaMemcpy(&st, status, 4, cudaMemcpyDeviceToHost));
          double bytes_cta = double(p.iters) * p.stage_bytes;
          printf("%-24s S=%d G=%3d  %7.3f ms  ingress/SM %6.1f GB/s  aggregate %6.2f TB/s  status %u\n",
                 mname[mi], sdepth, g, ms, bytes_cta / (ms * 1e6), bytes_cta * g / (ms * 1e9), st);
          if (st) { printf("status set, stopping\n"); return 2; }
        }
      }
    }
    // forwarding through distributed shared memory (CTA pairs), 32 KB stages
    const char* fname[] = {"pair: A forwarded", "pair: DSMEM only"};
    p.stage_bytes = STAGE;
    for (int mode = 1; mode <= 2; ++mode) {
      if (sh == 1 && mode == 2) continue;
      for (int g : grids) {
        p.mode = mode; p.iters = 6144;
        cudaLaunchConfig_t cfg{}; cfg.gridDim = dim3(g); cfg.blockDim = dim3(32);
        cfg.dynamicSmemBytes = 200 * 1024; cfg.stream = 0;
        cudaLaunchAttribute at[1]; at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 2; at[0].val.clusterDim.y = 1; at[0].val.clusterDim.z = 1;
        cfg.attrs = at; cfg.numAttrs = 1;
        float ms = 0;
        for (int rep = 0; rep < 2; ++rep) {
          CK(cudaEventRecord(e0));
          CK(cudaLaunchKernelEx(&cfg, probe<6>, p));
          CK(cudaEventRecord(e1));
          CK(cudaEventSynchronize(e1));
        }
        CK(cudaEventElapsedTime(&ms, e0, e1));
        unsigned int st; CK(cudaMemcpy(&st, status, 4, cudaMemcpyDeviceToHost));
        // bytes landed in the receiving CTA (rank 1) of each pair
        const double recv = double(p.iters) * (mode == 2 ? HALF : STAGE);
        printf("%-24s S=6 G=%3d  %7.3f ms  ingress of the receiving SM %6.1f GB/s  status %u\n",
               fname[mode - 1], g, ms, recv / (ms * 1e6), st);
        if (st) { printf("status set, stopping\n"); return 2; }
      }
    }
  }
  return 0;
}
