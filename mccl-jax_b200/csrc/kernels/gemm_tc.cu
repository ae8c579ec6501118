// gemm_tc.cu — dot_general on the B200 tensor cores: C[b] = A[b] . B[b]^T with A[b] (M x K) and
// B[b] (N x K), each stored K-major ([rows, K], K contiguous) or MN-major ([K, rows], rows
// contiguous), bf16 or f16, fp32 accumulation in TMEM, f32 / bf16 / f16 result.
//
// This replaces the reference's MPSGraph matmul call (src/jam/ops/linalg.mm:98, reached from
// DotGeneral linalg.mm:47-105 after its [batch, free, contract] canonicalisation).
//
// Design (one CTA per SM, persistent over output tiles of 128 x BN):
//   warp 0     TMA producer: 128x64 A and BNx64 B tiles (128-byte swizzle) into a kStages ring; an
//              MN-major operand arrives as 64(MN) x 64(K) boxes, 8 KB apart (the descriptor's LBO);
//   warp 1     allocates TMEM (2 x BN columns: double-buffered accumulator) and one thread issues
//              tcgen05.mma (M=128, N=BN, K=16) x4 per stage, committing stage release / acc-ready;
//   warps 2-5  epilogue: tcgen05.ld 32 lanes x 16 columns, convert, store; release the accumulator
//              so the next tile's MMAs overlap this tile's stores.
// Tails in M / N / K are handled by TMA zero fill and predicated stores.
#include <cuda_bf16.h>
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "kernels.h"
#include "tc_common.cuh"
#include "../../../include/b200_kernels.h"

namespace b200k {

static __device__ int g_tc_error_gemm;

namespace {

constexpr int BM = 128, BK = 64;
constexpr int kUnitRing = 4;   // work units published ahead by the TMA warp

// PAIR: the CTA is one of a pair (cluster of two) that computes 256 x BN tiles with M = 256
// tcgen05.mma over both CTAs (cta_group::2): each CTA loads 128 rows of A and BN / 2 rows of B, and
// holds its 128 x BN half of the accumulator in its own tensor memory.
template <int BN, bool PAIR = false>
struct Cfg {
  static constexpr int kBRows = PAIR ? BN / 2 : BN;        // B rows this CTA loads per stage
  static constexpr int kStages = BN == 256 ? (PAIR ? 6 : 4) : BN == 192 ? 5 : 6;
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = kBRows * BK * 2;
  static constexpr int kStage = kABytes + kBBytes;
  // epilogue staging (1024-byte aligned): 4 warps x 32 x 33 f32 for the bounds-checked path, or 4 x
  // 4 KB swizzled boxes for the TMA-store path
  static constexpr int kStageOut = 4 * 32 * 33 * 4;
  static constexpr int kSmem = kStages * kStage + 1024 + 1024 + kStageOut;
  static constexpr int kTmemCols = BN == 192 ? 512 : 2 * BN;   // allocations are powers of two
};

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
               ::"l"(map), "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4}], [%1];"
               ::"l"(map), "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Output tile order within a batch: bands of kGroupM row blocks, column-major inside a band.  The
// CTAs working at the same time (consecutive tile indices) then share a few A row blocks and B
// column blocks, which stay in L2, instead of streaming all of A once per B column block.
constexpr int kGroupM = 16;
__device__ __forceinline__ void tile_coords(int r, int mb, int nb, int* m_blk, int* n_blk) {
  const int band = r / (kGroupM * nb), first = band * kGroupM;
  const int rows = min(mb - first, kGroupM);
  const int q = r - band * kGroupM * nb;
  *m_blk = first + q % rows;
  *n_blk = q / rows;
}

// OUT: 0 f32, 1 bf16, 2 f16; AMN / BMN: operand stored MN-major; PAIR: see Cfg
template <int BN, int OUT, bool AMN, bool BMN, bool PAIR>
__global__ void __launch_bounds__(192, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, void* __restrict__ C, int M, int N, int K, int batch, int fmt,
               int splits, float* __restrict__ ws, int tma_store, long long ldc, int terms, uint32_t piece_a,
               uint32_t piece_b, int* __restrict__ unit_counter) {
  using CF = Cfg<BN, PAIR>;
  constexpr int TM = PAIR ? 2 * BM : BM;       // output rows per tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(smem + CF::kStages * CF::kStage);
  uint64_t* empty = full + CF::kStages;
  uint64_t* acc_full = empty + CF::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* unit_full = acc_empty + 2;         // ring of the work units this CTA processes
  uint64_t* unit_empty = unit_full + kUnitRing;
  int* unit_ring = (int*)(unit_empty + kUnitRing);
  uint32_t* tmem_slot = (uint32_t*)(unit_ring + kUnitRing);
  float* stage_base = (float*)(smem + CF::kStages * CF::kStage + 1024);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // in a pair the even CTA (rank 0) issues the MMAs and owns the full / acc_empty barriers
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const int unit0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int unit_step = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  // A pair drawing units from the counter: the even CTA claims them and writes each into both CTAs'
  // rings; the odd CTA's ring readers (its producer, MMA thread and epilogue warps) wait on their own
  // ring barrier (arrived on by the even CTA) and release the slot on the even CTA's barrier.
  const bool handoff = PAIR && unit_counter != nullptr;
  const bool ring_remote = handoff && rank != 0;
  auto ring_wait = [&](int rq, uint32_t parity, int code) {
    return ring_remote ? mbar_wait_cluster(&unit_full[rq], parity, code, &g_tc_error_gemm)
                       : mbar_wait(&unit_full[rq], parity, code, &g_tc_error_gemm);
  };
  auto ring_release = [&](int rq) {
    if (ring_remote) mbar_arrive_remote(cluster_addr(&unit_empty[rq], 0));
    else mbar_arrive(&unit_empty[rq]);
  };
  const int mb = (M + TM - 1) / TM, nb = (N + BN - 1) / BN;
  const int per_batch = mb * nb, num_tiles = per_batch * batch;
  // `terms` products accumulate into one result (the f32-accurate split form; 1 otherwise): term t
  // reads A's K piece (piece_a >> 4t) & 15 and B's (piece_b >> 4t) & 15, pieces sitting kbt K
  // blocks apart along K.  The K loop runs over terms x kbt blocks.
  const int kbt = (K + BK - 1) / BK;
  const int kbs = kbt * terms;
  // split-K: work unit u = (tile u / splits, K slice u % splits); slices are non-empty by construction
  // (host side), partial sums go to the f32 workspace through atomics
  const int kps = (kbs + splits - 1) / splits;
  const int num_units = num_tiles * splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < CF::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], PAIR ? 256 : 128);   // every epilogue thread (of both CTAs in a pair)
    }
    for (int q = 0; q < kUnitRing; ++q) {
      mbar_init(&unit_full[q], 1);
      // the MMA thread and the four epilogue warps (with a handoff: of both CTAs, and the odd CTA's
      // producer)
      mbar_init(&unit_empty[q], handoff ? 2 * (1 + 4) + 1 : 1 + 4);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    if (PAIR) tmem_alloc_pair(tmem_slot, CF::kTmemCols);
    else tmem_alloc(tmem_slot, CF::kTmemCols);
  }
  tc_fence_before();
  if (PAIR) cluster_sync();                    // the peer's barriers exist before anything signals them
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued = 0;  // bit s: stage s has a fill in flight of parity (ph_of_fill[s])
      uint32_t fill_par = 0;
      bool ok = true;
      // Work units come from the launch's counter when there is one: a CTA that starts late (its
      // SM held by another kernel, e.g. a collective) finds the units taken and leaves at once
      // instead of holding the launch back; the next unit is claimed while this one's loads are
      // issued, so the atomic's latency stays off the critical path.  Without a counter a CTA takes
      // every gridDim.x-th unit.  Each unit index, and finally one past the end, is published to
      // the MMA and epilogue warps through the ring.
      // (without a counter a pair walks the units statically: both CTAs take the same ones)
      int next = unit_counter ? (ring_remote ? 0 : atomicAdd(unit_counter, 1)) : unit0;
      for (int iu = 0;; ++iu) {
        const int rq = iu % kUnitRing;
        int u;
        if (ring_remote) {
          if (!ring_wait(rq, (iu / kUnitRing) & 1, kErrTimeoutEmpty)) break;
          u = *(volatile int*)&unit_ring[rq];
          ring_release(rq);
          if (u >= num_units) break;
        } else {
          u = ok ? next : num_units;
          if (handoff) {
            if (!mbar_wait_cluster(&unit_empty[rq], ((iu / kUnitRing) & 1) ^ 1, kErrTimeoutEmpty, &g_tc_error_gemm)) break;
            *(volatile int*)&unit_ring[rq] = u;
            st_cluster_u32(cluster_addr(&unit_ring[rq], 1), (uint32_t)u);
            mbar_arrive(&unit_full[rq]);
            mbar_arrive_remote(cluster_addr(&unit_full[rq], 1));
          } else {
            if (!mbar_wait(&unit_empty[rq], ((iu / kUnitRing) & 1) ^ 1, kErrTimeoutEmpty, &g_tc_error_gemm)) break;
            *(volatile int*)&unit_ring[rq] = u;
            mbar_arrive(&unit_full[rq]);
          }
          if (u >= num_units) break;
          next = unit_counter ? atomicAdd(unit_counter, 1) : u + unit_step;
        }
        const int t = u / splits, sp = u % splits;
        const int b = t / per_batch, r = t % per_batch;
        int m_blk, n_blk;
        tile_coords(r, mb, nb, &m_blk, &n_blk);
        const int kb1 = min(kbs, (sp + 1) * kps);
        for (int kb = sp * kps; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, kErrTimeoutEmpty, &g_tc_error_gemm)) { ok = false; break; }
          // a pair's loads all complete on the even CTA's full barrier, armed there for both
          if (!PAIR) mbar_arrive_expect_tx(&full[s], CF::kStage);
          else if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * CF::kStage);
          const uint32_t fbar = PAIR ? cluster_addr(&full[s], 0) : 0u;
          auto load = [&](const CUtensorMap* map, void* dst, int c0, int c1) {
            if (PAIR) tma_load_3d_pair(map, fbar, dst, c0, c1, b);
            else tma_load_3d(map, &full[s], dst, c0, c1, b);
          };
          uint8_t* sa = smem + s * CF::kStage;
          const int term = kb / kbt, kk = (kb - term * kbt) * BK;
          const int ka = (int)((piece_a >> (4 * term)) & 15u) * kbt * BK + kk;
          const int kb_ = (int)((piece_b >> (4 * term)) & 15u) * kbt * BK + kk;
          const int a_row = m_blk * TM + (int)rank * BM, b_row = n_blk * BN + (int)rank * CF::kBRows;
          if (AMN) {
#pragma unroll
            for (int i = 0; i < BM / 64; ++i) load(&tmA, sa + i * 8192, a_row + 64 * i, ka);
          } else {
            load(&tmA, sa, ka, a_row);
          }
          if (BMN) {
#pragma unroll
            for (int i = 0; i < CF::kBRows / 64; ++i) load(&tmB, sa + CF::kABytes + i * 8192, b_row + 64 * i, kb_);
          } else {
            load(&tmB, sa + CF::kABytes, kb_, b_row);
          }
          issued |= 1u << s;
          fill_par = (fill_par & ~(1u << s)) | (ph << s);
          if (++s == CF::kStages) { s = 0; ph ^= 1; }
        }
      }
      // never leave with TMA writes in flight: wait (bounded) for the last fill of every stage (in a
      // pair the even CTA's full barriers count both CTAs' loads; the odd CTA stays until the pair's
      // final cluster barrier, which the even CTA reaches after this wait)
      if (rank == 0)
        for (int q = 0; q < CF::kStages; ++q)
          if (issued & (1u << q)) mbar_wait(&full[q], (fill_par >> q) & 1, kErrTimeoutOther, &g_tc_error_gemm);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(fmt, TM, BN, BMN, AMN);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int local = 0; ok; ++local) {
        const int rq = local % kUnitRing;
        if (!ring_wait(rq, (local / kUnitRing) & 1, kErrTimeoutFull)) break;
        const int u = *(volatile int*)&unit_ring[rq];
        ring_release(rq);
        if (u >= num_units) break;
        if (rank != 0) continue;                 // the odd CTA of a pair issues no MMAs
        const int a = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[a], aph ^ 1, kErrTimeoutAccEmpty, &g_tc_error_gemm)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + a * BN;
        const int sp = u % splits, kb0 = sp * kps, kb1 = min(kbs, (sp + 1) * kps);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[s], ph, kErrTimeoutFull, &g_tc_error_gemm)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * CF::kStage);
          const uint32_t b_addr = a_addr + CF::kABytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t da = AMN ? sw128_mn_desc_lbo(a_addr + k * 2048, 8192) : sw128_desc(a_addr + k * 32);
            const uint64_t db = BMN ? sw128_mn_desc_lbo(b_addr + k * 2048, 8192) : sw128_desc(b_addr + k * 32);
            if (PAIR) mma_f16_ss_pair(d, da, db, idesc, ((kb - kb0) | k) != 0);
            else mma_f16_ss(d, da, db, idesc, ((kb - kb0) | k) != 0);
          }
          if (PAIR) mma_commit_pair(&empty[s]);  // frees the stage in both CTAs
          else mma_commit(&empty[s]);
          if (++s == CF::kStages) { s = 0; ph ^= 1; }
        }
        if (ok) {
          if (PAIR) mma_commit_pair(&acc_full[a]);
          else mma_commit(&acc_full[a]);
        }
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    // the accumulator buffer is free again once every epilogue thread (of both CTAs in a pair) has
    // read its part; a pair's MMAs wait on the even CTA's barrier
    auto release_acc = [&](int a) {
      if (PAIR && rank != 0) mbar_arrive_remote(cluster_addr(&acc_empty[a], 0));
      else mbar_arrive(&acc_empty[a]);
    };
    for (int local = 0;; ++local) {
      const int rq = local % kUnitRing;
      if (!__all_sync(0xffffffffu, ring_wait(rq, (local / kUnitRing) & 1, kErrTimeoutAcc))) break;
      const int u = *(volatile int*)&unit_ring[rq];
      __syncwarp();
      if (lane == 0) ring_release(rq);
      if (u >= num_units) break;
      const int t = u / splits;
      const int a = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!mbar_wait_warp(&acc_full[a], aph, kErrTimeoutAcc, &g_tc_error_gemm)) break;
      tc_fence_after();
      const int b = t / per_batch, r = t % per_batch;
      int m_blk, n_blk;
      tile_coords(r, mb, nb, &m_blk, &n_blk);
      const int m0 = m_blk * TM + (int)rank * BM;   // first output row of this CTA's accumulator half
      const int row = m0 + row_in_tile;
      const uint32_t taddr = tmem_base + a * BN + ((uint32_t)(q * 32) << 16);
      const long long crow = ((long long)b * M + row) * ldc;      // ldc: C's row pitch (>= N)
      // full 32-column chunks of an aligned row go straight out as 16-byte vectors; otherwise (N not
      // a multiple of 8 / 4, or the ragged last chunk) the warp stages 32 rows x 32 columns in shared
      // memory and writes them row by row, coalesced, with bounds checks
      const bool aligned = OUT == 0 ? (ldc & 3) == 0 : (ldc & 7) == 0;
      float* stage = stage_base + (warp - 2) * 32 * 33;
      if (tma_store == 2) {
        // split-K partial sums: f32 boxes added into the workspace by TMA reduce-add (L2 atomics
        // on whole lines instead of one per element)
        uint8_t* box = (uint8_t*)stage_base + (warp - 2) * 4096;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t v[32];
          tmem_ld16(taddr + c, *reinterpret_cast<uint32_t(*)[16]>(v));
          tmem_ld16(taddr + c + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
          tmem_wait_ld();
          const int col = n_blk * BN + c;
          if (col >= N) continue;                      // warp-uniform
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 8; ++i)
            *(uint4*)(box + lane * 128 + ((i ^ (lane & 7)) << 4)) = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_reduce_add_3d(&tmC, box, col, m0 + q * 32, b);
            bulk_commit();
          }
        }
        tc_fence_before();
        release_acc(a);
        continue;
      }
      if (tma_store) {
        // 128-byte rows (32 f32 or 64 16-bit columns) into a 128-byte-swizzled 32-row box, written out
        // by one TMA store per chunk (full-line writes; M / N tails clipped by the tensor map)
        uint8_t* box = (uint8_t*)stage_base + (warp - 2) * 4096;
        constexpr int CW = OUT == 0 ? 32 : 64;
#pragma unroll 1
        for (int c = 0; c < BN; c += CW) {
          uint32_t v[CW];
#pragma unroll
          for (int j = 0; j < CW; j += 16) tmem_ld16(taddr + c + j, *reinterpret_cast<uint32_t(*)[16]>(v + j));
          tmem_wait_ld();
          const int col = n_blk * BN + c;
          if (col >= N) continue;                      // warp-uniform
          uint32_t w[32];
#pragma unroll
          for (int j = 0; j < 32; ++j)
            w[j] = OUT == 0 ? v[j]
                 : OUT == 1 ? pack_bf16(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]))
                            : pack_f16(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
          if (lane == 0) bulk_wait_read0();            // the previous store has read the box
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 8; ++i)
            *(uint4*)(box + lane * 128 + ((i ^ (lane & 7)) << 4)) = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tmC, box, col, m0 + q * 32, b);
            bulk_commit();
          }
        }
        tc_fence_before();
        release_acc(a);
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t v[32];
        tmem_ld16(taddr + c, *reinterpret_cast<uint32_t(*)[16]>(v));
        tmem_ld16(taddr + c + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
        tmem_wait_ld();
        const int col = n_blk * BN + c;
        if (col >= N) continue;                        // warp-uniform
        if (splits > 1) {
          // partial sum of one K slice: f32 atomics into the workspace, coalesced through the stage
#pragma unroll
          for (int j = 0; j < 32; ++j) stage[lane * 33 + j] = __uint_as_float(v[j]);
          __syncwarp();
          const int gcol = col + lane;
#pragma unroll 4
          for (int rr = 0; rr < 32; ++rr) {
            const int grow = m0 + q * 32 + rr;
            if (grow < M && gcol < N) atomicAdd(ws + ((long long)b * M + grow) * (long long)N + gcol, stage[rr * 33 + lane]);
          }
          __syncwarp();
        } else if (aligned && col + 32 <= N) {
          if (row < M) {
            if (OUT == 0) {
              float* out = (float*)C + crow + col;
#pragma unroll
              for (int j = 0; j < 32; j += 4)
                *(float4*)(out + j) = make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                                                  __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
            } else {
              uint16_t* out = (uint16_t*)C + crow + col;
              uint32_t p[16];
#pragma unroll
              for (int j = 0; j < 16; ++j)
                p[j] = OUT == 1 ? pack_bf16(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]))
                                : pack_f16(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
#pragma unroll
              for (int j = 0; j < 16; j += 4) *(uint4*)(out + 2 * j) = make_uint4(p[j], p[j + 1], p[j + 2], p[j + 3]);
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) stage[lane * 33 + j] = __uint_as_float(v[j]);
          __syncwarp();
          const int gcol = col + lane;
#pragma unroll 4
          for (int rr = 0; rr < 32; ++rr) {
            const int grow = m0 + q * 32 + rr;
            if (grow < M && gcol < N) {
              const float x = stage[rr * 33 + lane];
              const long long o = ((long long)b * M + grow) * ldc + gcol;
              if (OUT == 0) ((float*)C)[o] = x;
              else if (OUT == 1) ((uint16_t*)C)[o] = (uint16_t)(pack_bf16(x, 0.f) & 0xffff);
              else ((uint16_t*)C)[o] = (uint16_t)(pack_f16(x, 0.f) & 0xffff);
            }
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      release_acc(a);
    }
  }
  if (warp >= 2 && lane == 0) bulk_wait_all();    // TMA stores complete before the CTA's smem goes away
  tc_fence_before();
  if (PAIR) cluster_sync();                      // neither CTA leaves while the pair's MMAs may read it
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR) tmem_dealloc_pair(tmem_base, CF::kTmemCols);
    else tmem_dealloc(tmem_base, CF::kTmemCols);
  }
}

// ---------------------------------------------------------------------------- SIMT fallback
// fp32 (or any) inputs, A[b] (M x K) and B[b] (N x K), each K-major (row pitch ld) or MN-major ([K,
// rows], pitch ld): 128x128 tiles, 8x8 outputs per thread.
template <typename T, int OUT, bool AMN, bool BMN>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const T* __restrict__ A, const T* __restrict__ B, void* __restrict__ C,
                                                        int M, int N, int K, long long lda, long long ldb) {
  __shared__ float As[16][128 + 4];
  __shared__ float Bs[16][128 + 4];
  const int b = blockIdx.z;
  const int m0 = blockIdx.y * 128, n0 = blockIdx.x * 128;
  const T* Ab = A + (long long)b * (AMN ? K : M) * lda;
  const T* Bb = B + (long long)b * (BMN ? K : N) * ldb;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  for (int k0 = 0; k0 < K; k0 += 16) {
    // 128 rows x 16 k per operand = 2048 elements; 256 threads x 8
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      int idx = threadIdx.x + e * 256;
      {
        int row = AMN ? idx & 127 : idx >> 4, kk = AMN ? idx >> 7 : idx & 15;
        int gk = k0 + kk, gm = m0 + row;
        As[kk][row] = (gm < M && gk < K) ? (float)Ab[AMN ? (long long)gk * lda + gm : (long long)gm * lda + gk] : 0.f;
      }
      {
        int row = BMN ? idx & 127 : idx >> 4, kk = BMN ? idx >> 7 : idx & 15;
        int gk = k0 + kk, gn = n0 + row;
        Bs[kk][row] = (gn < N && gk < K) ? (float)Bb[BMN ? (long long)gk * ldb + gn : (long long)gn * ldb + gk] : 0.f;
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float av[8], bv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) av[i] = As[kk][ty * 8 + i];
#pragma unroll
      for (int j = 0; j < 8; ++j) bv[j] = Bs[kk][tx * 8 + j];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int gm = m0 + ty * 8 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int gn = n0 + tx * 8 + j;
      if (gn >= N) continue;
      long long o = ((long long)b * M + gm) * N + gn;
      if (OUT == 0) ((float*)C)[o] = acc[i][j];
      else if (OUT == 1) ((__nv_bfloat16*)C)[o] = __float2bfloat16_rn(acc[i][j]);
      else ((__half*)C)[o] = __float2half_rn(acc[i][j]);
    }
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

}  // namespace

EncodeTiledFn GetEncodeTiled();

// 3-D K-major operand map: dims {K, rows, batch} with row pitch `ld` elements (ld * 2 % 16 == 0),
// box {64, box_rows, 1}, 128-byte swizzle.  Columns K .. ld-1 are never read (zero fill past K).
bool MakeOperandMap(CUtensorMap* map, const void* ptr, int K, long long ld, int rows, int batch, int box_rows,
                    bool f16like) {
  EncodeTiledFn enc = GetEncodeTiled();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)ld * 2 * rows};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, f16like ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr),
                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 3-D MN-major operand map: dims {rows, K, batch} with K-row pitch `ld` elements (ld * 2 % 16 == 0),
// box {64, 64, 1} (64 MN elements = one 128-byte swizzle row, 64 k), 128-byte swizzle.
bool MakeOperandMapMN(CUtensorMap* map, const void* ptr, int K, long long ld, int rows, int batch, bool f16like) {
  EncodeTiledFn enc = GetEncodeTiled();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)rows, (cuuint64_t)K, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)ld * 2 * K};
  cuuint32_t box[3] = {64, 64, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, f16like ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr),
                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 3-D output map for the TMA-store epilogue: dims {N, M, batch}, box {128 bytes of columns, 32 rows, 1},
// 128-byte swizzle.  Rows must be 16-byte multiples.
bool MakeOutputMap(CUtensorMap* map, void* C, int M, int N, int batch, int out, long long ldc) {
  EncodeTiledFn enc = GetEncodeTiled();
  if (!enc) return false;
  const int esz = out == 0 ? 4 : 2;
  cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)M, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)ldc * esz, (cuuint64_t)ldc * esz * M};
  cuuint32_t box[3] = {(cuuint32_t)(128 / esz), 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMapDataType t = out == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : out == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return enc(map, t, 3, C, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int NumSMs() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

// Operand K extents of the tensor maps and the term table of a launch (see gemm_tc_kernel): plain
// products read one piece per operand whose map spans K; the split form reads pieces side by side.
struct Terms {
  int n = 1;
  uint32_t a = 0, b = 0;     // 4 bits per term: the piece index of A / B
  long long ka = -1, kb = -1;  // K extent of A's / B's map (-1: K)
};

// CTA pairs (clusters of two) of the pair kernel that fit on the device at once; 0 if none.
template <int BN, int OUT, bool AMN, bool BMN>
static int MaxPairs() {
  static int pairs[8] = {-1, -1, -1, -1, -1, -1, -1, -1};
  int dev = 0;
  cudaGetDevice(&dev);
  int& p = pairs[dev & 7];
  if (p < 0) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * NumSMs());
    cfg.blockDim = dim3(192);
    cfg.dynamicSmemBytes = Cfg<BN, true>::kSmem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel<BN, OUT, AMN, BMN, true>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    p = n;
  }
  return p;
}

template <int BN, int OUT, bool AMN, bool BMN, bool PAIR>
static int LaunchTc(const void* A, long long lda, const void* B, long long ldb, void* C, int batch, int M, int N, int K,
                    int fmt, cudaStream_t st, int splits, float* ws, long long ldc, const Terms& tm, int* counter) {
  using CF = Cfg<BN, PAIR>;
  static std::once_flag once[8];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 7], [] {
    cudaFuncSetAttribute(gemm_tc_kernel<BN, OUT, AMN, BMN, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize, CF::kSmem);
  });
  CUtensorMap ta, tb, tc;
  const int ka = tm.ka < 0 ? K : (int)tm.ka, kb = tm.kb < 0 ? K : (int)tm.kb;
  bool ok = AMN ? MakeOperandMapMN(&ta, A, ka, lda, M, batch, fmt == 0) : MakeOperandMap(&ta, A, ka, lda, M, batch, BM, fmt == 0);
  ok = ok && (BMN ? MakeOperandMapMN(&tb, B, kb, ldb, N, batch, fmt == 0)
                  : MakeOperandMap(&tb, B, kb, ldb, N, batch, CF::kBRows, fmt == 0));
  if (!ok) return -2;
  // TMA-store epilogue when C's rows are 16-byte multiples (else the bounds-checked staged path);
  // split-K partials go to the f32 workspace by TMA reduce-add under the same condition
  const int esz = OUT == 0 ? 4 : 2;
  int tma_store = 0;
  if (!getenv("B200_GEMM_NO_TMA_STORE")) {
    if (splits == 1 && (ldc * esz) % 16 == 0 && ((uintptr_t)C % 16) == 0)
      tma_store = MakeOutputMap(&tc, C, M, N, batch, OUT, ldc) ? 1 : 0;
    else if (splits > 1 && ((long long)N * 4) % 16 == 0 && ((uintptr_t)ws % 16) == 0)
      tma_store = MakeOutputMap(&tc, ws, M, N, batch, 0, N) ? 2 : 0;
  }
  if (!tma_store) tc = ta;                                  // unused
  constexpr int TM = PAIR ? 2 * BM : BM;
  const int tiles = ((M + TM - 1) / TM) * ((N + BN - 1) / BN) * batch;
  if constexpr (!PAIR) {
    const int grid = std::min(tiles * splits, NumSMs());
    gemm_tc_kernel<BN, OUT, AMN, BMN, false><<<grid, 192, CF::kSmem, st>>>(ta, tb, tc, C, M, N, K, batch, fmt, splits, ws,
                                                                           tma_store, ldc, tm.n, tm.a, tm.b, counter);
  } else {
    const int pairs = std::min(tiles * splits, MaxPairs<BN, OUT, AMN, BMN>());
    if (pairs < 1) return -3;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(192);
    cfg.dynamicSmemBytes = CF::kSmem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN, OUT, AMN, BMN, true>, ta, tb, tc, C, M, N, K, batch, fmt, splits, ws,
                           tma_store, ldc, tm.n, tm.a, tm.b, counter) != cudaSuccess)
      return -3;
  }
  CountLaunches();
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

template <int BN, int OUT, bool PAIR>
static int LaunchTcMajor(bool amn, bool bmn, const void* A, long long lda, const void* B, long long ldb, void* C, int batch,
                         int M, int N, int K, int fmt, cudaStream_t st, int splits, float* ws, long long ldc,
                         const Terms& tm, int* counter) {
  if (amn && bmn) return LaunchTc<BN, OUT, true, true, PAIR>(A, lda, B, ldb, C, batch, M, N, K, fmt, st, splits, ws, ldc, tm, counter);
  if (amn) return LaunchTc<BN, OUT, true, false, PAIR>(A, lda, B, ldb, C, batch, M, N, K, fmt, st, splits, ws, ldc, tm, counter);
  if (bmn) return LaunchTc<BN, OUT, false, true, PAIR>(A, lda, B, ldb, C, batch, M, N, K, fmt, st, splits, ws, ldc, tm, counter);
  return LaunchTc<BN, OUT, false, false, PAIR>(A, lda, B, ldb, C, batch, M, N, K, fmt, st, splits, ws, ldc, tm, counter);
}

__global__ void __launch_bounds__(256) ws_to_16bit_kernel(const float* __restrict__ ws, uint16_t* __restrict__ c, long long n,
                                                           int f16) {
  for (long long i = (long long)blockIdx.x * 256 + threadIdx.x; i < n; i += (long long)gridDim.x * 256)
    c[i] = (uint16_t)((f16 ? pack_f16(ws[i], 0.f) : pack_bf16(ws[i], 0.f)) & 0xffff);
}

template <typename T, bool AMN, bool BMN>
static int LaunchSimtT(const void* A, long long lda, const void* B, long long ldb, void* C, int batch, int M, int N, int K,
                       int out, cudaStream_t st) {
  dim3 grid((N + 127) / 128, (M + 127) / 128, batch);
  if (out == 0) gemm_simt_kernel<T, 0, AMN, BMN><<<grid, 256, 0, st>>>((const T*)A, (const T*)B, C, M, N, K, lda, ldb);
  else if (out == 1) gemm_simt_kernel<T, 1, AMN, BMN><<<grid, 256, 0, st>>>((const T*)A, (const T*)B, C, M, N, K, lda, ldb);
  else gemm_simt_kernel<T, 2, AMN, BMN><<<grid, 256, 0, st>>>((const T*)A, (const T*)B, C, M, N, K, lda, ldb);
  CountLaunches();
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

template <typename T>
static int LaunchSimt(bool amn, bool bmn, const void* A, long long lda, const void* B, long long ldb, void* C, int batch,
                      int M, int N, int K, int out, cudaStream_t st) {
  if (amn && bmn) return LaunchSimtT<T, true, true>(A, lda, B, ldb, C, batch, M, N, K, out, st);
  if (amn) return LaunchSimtT<T, true, false>(A, lda, B, ldb, C, batch, M, N, K, out, st);
  if (bmn) return LaunchSimtT<T, false, true>(A, lda, B, ldb, C, batch, M, N, K, out, st);
  return LaunchSimtT<T, false, false>(A, lda, B, ldb, C, batch, M, N, K, out, st);
}

int TakeGemmError() {
  int v = 0, z = 0;
  cudaMemcpyFromSymbol(&v, g_tc_error_gemm, sizeof(int));
  if (v) cudaMemcpyToSymbol(g_tc_error_gemm, &z, sizeof(int));
  return v;
}

// C[b] = A[b] . B[b]^T.  A is [batch, M, >=K] (K-major, row pitch lda) or, with a_mn, [batch, K, >=M]
// (MN-major, pitch lda); B likewise with N, ldb and b_mn.
// Tile width and K slices for a tensor-core GEMM, chosen by a wave model: the time of a persistent
// launch is the number of rounds of work units over the SMs times the time of one unit, which grows
// with the tile width (BN = 256, 192 or 128 columns) and the unit's K blocks plus about two blocks of
// fill and epilogue; narrower tiles pay a little for feeding the tensor cores more operand bytes
// per FLOP.  K is split (at most 8 slices of >= 16 K blocks, none empty) when that shortens the
// model's time including the f32 partials' cost (a zeroing pass, L2 reductions and, for 16-bit
// results, a rounding pass): when the tiles leave SMs idle, or when a long K walk makes the last
// round of tiles a large fraction of the launch.  256-column tiles may also run on CTA pairs (256 x
// 256 tiles on two SMs, half the shared-memory operand traffic per SM: measured 12-19 % faster per
// tile on B200), which halves the tile count and the units' slots.  Shared by the compiler (which
// sizes the workspace) and the launcher.  B200_GEMM_PAIR=0 / 1 turns pairs off / forces them for
// every 256-column choice.
void GemmTile(int64_t batch, int64_t M, int64_t N, int64_t K, int sms, int* bn_out, int* splits_out, bool* pair_out) {
  const int64_t kbs = std::max<int64_t>(1, (K + BK - 1) / BK);
  const bool no_split = std::getenv("B200_GEMM_NO_SPLITK") != nullptr || K <= 0;
  const char* force = std::getenv("B200_GEMM_BN");
  const char* pair_env = std::getenv("B200_GEMM_PAIR");
  const bool pair_off = pair_env && pair_env[0] == '0', pair_forced = pair_env && pair_env[0] == '1';
  double best = 1e300;
  int best_bn = 256, best_s = 1;
  bool best_pair = false;
  for (int bn : {256, 192, 128}) {
    if (force && std::atoi(force) != bn) continue;
    if (!force && bn > 128 && N < bn) continue;
    for (int pair = 0; pair <= (bn == 256 ? 1 : 0); ++pair) {
      if (pair ? (pair_off || M < 2 * BM) : (pair_forced && bn == 256 && M >= 2 * BM)) continue;
      const int64_t tm = pair ? 2 * BM : BM, slots = pair ? sms / 2 : sms;
      const int64_t tiles = ((M + tm - 1) / tm) * ((N + bn - 1) / bn) * batch;
      const double width = pair ? 0.85 : bn / 256.0 * (bn == 128 ? 1.3 : bn == 192 ? 1.08 : 1.0);   // measured on B200
      for (int64_t s = 1; s <= 8; ++s) {
        if (s > 1 && (no_split || kbs / s < 16 || (tiles * 2 > slots && kbs < 128))) break;
        const int64_t kps = (kbs + s - 1) / s;
        if (s > 1 && (s - 1) * kps >= kbs) continue;        // would leave an empty slice
        const int64_t rounds = (tiles * s + slots - 1) / slots;
        double t = (double)rounds * width * (double)(kps + 2);
        // splitting: zero + reduce + round the f32 partials, ~10 bytes per output at HBM speed, in
        // units of one 128 x 256 x 64 block step (~0.45 us)
        if (s > 1) t += (double)batch * M * N * 10.0 / 6.5e12 / 0.45e-6;
        if (t < best * 0.999) { best = t; best_bn = bn; best_s = (int)s; best_pair = pair != 0; }
      }
    }
  }
  *bn_out = best_bn;
  *splits_out = best_s;
  if (pair_out) *pair_out = best_pair;
}

int GemmSplitK(int64_t batch, int64_t M, int64_t N, int64_t K, int sms) {
  int bn = 256, s = 1;
  GemmTile(batch, M, N, K, sms, &bn, &s);
  return s;
}

// Runs one tensor-core launch (tile width and K slices from the wave model over `k_eff` = the K
// blocks every output tile walks), plus the split-K zeroing and rounding passes.
static int RunTc(const void* A, long long lda, bool a_mn, const void* B, long long ldb, bool b_mn, void* C, int64_t batch,
                 int64_t M, int64_t N, int64_t K, int64_t k_eff, int fmt, int out, cudaStream_t st, float* ws, int64_t ldc,
                 const Terms& tm, int* counter) {
  int b = (int)batch, m = (int)M, n = (int)N, k = (int)K;
  int bn = 256, splits = 1;
  bool pair = false;
  GemmTile(batch, M, N, k_eff, NumSMs(), &bn, &splits, &pair);
  if (ldc != N) splits = 1;                  // partial sums are laid out densely
  float* acc = out == 0 ? (float*)C : ws;
  if (splits > 1 && !acc) splits = 1;
  if (splits > 1 && cudaMemsetAsync(acc, 0, (size_t)batch * M * N * 4, st) != cudaSuccess) return -3;
  auto launch = [&](auto out_c) {
    constexpr int O = decltype(out_c)::value;
    if (bn == 256 && pair)
      return LaunchTcMajor<256, O, true>(a_mn, b_mn, A, lda, B, ldb, C, b, m, n, k, fmt, st, splits, acc, ldc, tm, counter);
    if (bn == 256) return LaunchTcMajor<256, O, false>(a_mn, b_mn, A, lda, B, ldb, C, b, m, n, k, fmt, st, splits, acc, ldc, tm,
                                                         counter);
    if (bn == 192) return LaunchTcMajor<192, O, false>(a_mn, b_mn, A, lda, B, ldb, C, b, m, n, k, fmt, st, splits, acc, ldc, tm,
                                                         counter);
    return LaunchTcMajor<128, O, false>(a_mn, b_mn, A, lda, B, ldb, C, b, m, n, k, fmt, st, splits, acc, ldc, tm, counter);
  };
  int rc = out == 0 ? launch(std::integral_constant<int, 0>{})
         : out == 1 ? launch(std::integral_constant<int, 1>{})
                    : launch(std::integral_constant<int, 2>{});
  if (rc == 0 && splits > 1 && out != 0) {
    const long long total = (long long)batch * M * N;
    ws_to_16bit_kernel<<<(unsigned)std::min<long long>((total + 255) / 256, 148 * 8), 256, 0, st>>>(acc, (uint16_t*)C, total,
                                                                                                   out == 2);
    CountLaunches();
    rc = cudaGetLastError() == cudaSuccess ? 0 : -3;
  }
  return rc;
}

static int OutCode(int out_type) {
  return out_type == B200_DT_F32 ? 0 : out_type == B200_DT_BF16 ? 1 : out_type == B200_DT_F16 ? 2 : -1;
}

// C[b] = A[b] . B[b]^T.  A is [batch, M, >=K] (K-major, row pitch lda) or, with a_mn, [batch, K, >=M]
// (MN-major, pitch lda); B likewise with N, ldb and b_mn.  With `ws` (batch*M*N f32) a 16-bit result
// may be computed split-K (partials added into ws, then rounded into C); an f32 result splits without
// it (partials added into C).
int Gemm(const void* A, long long lda, bool a_mn, const void* B, long long ldb, bool b_mn, void* C, int64_t batch, int64_t M,
         int64_t N, int64_t K, int ab_type, int out_type, cudaStream_t st, float* ws, int64_t ldc, int* counter) {
  if (batch <= 0 || M <= 0 || N <= 0) return 0;
  if (ldc <= 0) ldc = N;
  if (ldc < N) return -1;
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX || batch > 65535 || lda < (a_mn ? M : K) || ldb < (b_mn ? N : K))
    return -1;
  const int out = OutCode(out_type);
  if (out < 0) return -1;
  if (K == 0) {
    size_t bytes = (size_t)batch * M * ldc * (out == 0 ? 4 : 2);
    return cudaMemsetAsync(C, 0, bytes, st) == cudaSuccess ? 0 : -3;
  }
  bool tc_ok = (ab_type == B200_DT_BF16 || ab_type == B200_DT_F16) && (lda % 8) == 0 && (ldb % 8) == 0 &&
               ((uintptr_t)A % 16) == 0 && ((uintptr_t)B % 16) == 0 && !getenv("B200_GEMM_SIMT");
  if (tc_ok)
    return RunTc(A, lda, a_mn, B, ldb, b_mn, C, batch, M, N, K, K, ab_type == B200_DT_BF16 ? 1 : 0, out, st, ws, ldc, Terms{},
                 counter);
  int b = (int)batch, m = (int)M, n = (int)N, k = (int)K;
  if (ldc != N) return -1;                     // padded C rows are written by the tensor-core path only
  if (ab_type == B200_DT_F32) return LaunchSimt<float>(a_mn, b_mn, A, lda, B, ldb, C, b, m, n, k, out, st);
  if (ab_type == B200_DT_BF16) return LaunchSimt<__nv_bfloat16>(a_mn, b_mn, A, lda, B, ldb, C, b, m, n, k, out, st);
  if (ab_type == B200_DT_F16) return LaunchSimt<__half>(a_mn, b_mn, A, lda, B, ldb, C, b, m, n, k, out, st);
  return -1;
}

int Gemm(const void* A, long long lda, const void* B, long long ldb, void* C, int64_t batch, int64_t M, int64_t N,
         int64_t K, int ab_type, int out_type, cudaStream_t st) {
  return Gemm(A, lda, false, B, ldb, false, C, batch, M, N, K, ab_type, out_type, st, nullptr, 0, nullptr);
}

// ---------------------------------------------------------------------------- f32-accurate products
namespace {

__device__ __forceinline__ float load_as_f32(const float* p) { return *p; }
__device__ __forceinline__ float load_as_f32(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ float load_as_f32(const __half* p) { return __half2float(*p); }

// bf16 pieces of an operand: element (b, k, r) of the logical [batch, K, rows] operand (src stored
// K-major [batch, rows, ld] or, with src_mn, MN-major [batch, K, ld]) gives `pieces` bf16 values
// h_j = bf16_rn(x - h_0 - ... - h_{j-1}) (each difference exact in f32), written to
//   dst_mn = 0: dst[b][r][j * Kp + k]      (K-major, pieces side by side along K)
//   dst_mn = 1: dst[b][j * Kp + k][r]      (MN-major)
// with zeros for k in [K, Kp).  Threads walk the destination (coalesced stores), 4 elements each.
template <typename T>
__global__ void __launch_bounds__(256) split_pieces_kernel(const T* __restrict__ src, long long ld, int src_mn, int dst_mn,
                                                           int batch, int rows, int K, int Kp, int pieces,
                                                           uint16_t* __restrict__ dst, int vec_ok) {
  const long long outer = dst_mn ? (long long)pieces * Kp : rows;      // destination rows per batch
  const long long inner = dst_mn ? rows : (long long)pieces * Kp;      // destination row length
  const long long quads = inner / 4;                                   // inner % 4 == 0 (host-checked)
  const long long total = (long long)batch * outer * quads;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
    const long long q = e % quads, t = e / quads;
    const long long o = t % outer, b = t / outer;
    uint16_t h[4];
    if (sizeof(T) == 4 && vec_ok && src_mn == dst_mn) {
      // same layout on both sides: the quad is 4 consecutive source elements of one piece, read as
      // one 16-byte load when they are all inside the operand
      const long long i = q * 4;
      long long j, k, r;
      if (dst_mn) { j = o / Kp; k = o - j * Kp; r = i; }
      else { j = i / Kp; k = i - j * Kp; r = o; }
      const bool inside = dst_mn ? (k < K) : (k + 3 < K);
      if (inside) {
        const float4 x4 = *reinterpret_cast<const float4*>(src + (src_mn ? (b * K + k) * ld + r : (b * rows + r) * ld + k));
        float xs[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          float x = xs[v];
          __nv_bfloat16 piece = __float2bfloat16_rn(x);
          for (long long p = 0; p < j; ++p) {
            x -= __bfloat162float(piece);
            piece = __float2bfloat16_rn(x);
          }
          h[v] = __bfloat16_as_ushort(piece);
        }
        *(uint2*)(dst + (b * outer + o) * inner + q * 4) =
            make_uint2((uint32_t)h[0] | ((uint32_t)h[1] << 16), (uint32_t)h[2] | ((uint32_t)h[3] << 16));
        continue;
      }
    }
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const long long i = q * 4 + v;
      // destination element -> (piece j, k, r)
      long long j, k, r;
      if (dst_mn) { j = o / Kp; k = o - j * Kp; r = i; }
      else { j = i / Kp; k = i - j * Kp; r = o; }
      float x = 0.f;
      if (k < K) x = load_as_f32(src + (src_mn ? (b * K + k) * ld + r : (b * rows + r) * ld + k));
      // peel pieces 0..j (each a round-to-nearest-even bf16 of the remainder)
      __nv_bfloat16 piece = __float2bfloat16_rn(x);
      for (long long p = 0; p < j; ++p) {
        x -= __bfloat162float(piece);
        piece = __float2bfloat16_rn(x);
      }
      h[v] = __bfloat16_as_ushort(piece);
    }
    *(uint2*)(dst + (b * outer + o) * inner + q * 4) =
        make_uint2((uint32_t)h[0] | ((uint32_t)h[1] << 16), (uint32_t)h[2] | ((uint32_t)h[3] << 16));
  }
}

// How an operand enters the split product: in place (a bf16 operand TMA can read) or as `pieces`
// bf16 pieces in scratch, K-major or MN-major.
struct SplitOperand {
  int pieces = 1;
  bool in_place = false;
  bool dst_mn = false;
  size_t bytes = 0;                            // scratch bytes
};

SplitOperand PlanOperand(int type, bool mn, long long ld, const void* ptr, int64_t batch, int64_t rows, int64_t Kp) {
  SplitOperand o;
  o.pieces = type == B200_DT_BF16 ? 1 : 3;     // f16 and f32 take three bf16 pieces
  o.in_place = type == B200_DT_BF16 && ld % 8 == 0 && ((uintptr_t)ptr % 16) == 0 && (!mn || rows % 8 == 0);
  o.dst_mn = mn && rows % 8 == 0;
  if (!o.in_place) o.bytes = ((size_t)batch * rows * o.pieces * Kp * 2 + 255) / 256 * 256;
  return o;
}

template <typename T>
int LaunchSplit(const void* src, long long ld, bool src_mn, const SplitOperand& o, int64_t batch, int64_t rows, int64_t K,
                int64_t Kp, void* dst, cudaStream_t st) {
  const long long total = (long long)batch * rows * o.pieces * Kp / 4;
  const int grid = (int)std::min<long long>((total + 255) / 256, (long long)NumSMs() * 8);
  // 16-byte source loads need a 16-byte aligned base and rows of a multiple of 4 elements
  const int vec_ok = ((uintptr_t)src % 16) == 0 && (ld % 4) == 0;
  split_pieces_kernel<T><<<grid, 256, 0, st>>>((const T*)src, ld, src_mn ? 1 : 0, o.dst_mn ? 1 : 0, (int)batch, (int)rows,
                                               (int)K, (int)Kp, o.pieces, (uint16_t*)dst, vec_ok);
  CountLaunches();
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int Split(int type, const void* src, long long ld, bool src_mn, const SplitOperand& o, int64_t batch, int64_t rows, int64_t K,
          int64_t Kp, void* dst, cudaStream_t st) {
  if (type == B200_DT_F32) return LaunchSplit<float>(src, ld, src_mn, o, batch, rows, K, Kp, dst, st);
  if (type == B200_DT_BF16) return LaunchSplit<__nv_bfloat16>(src, ld, src_mn, o, batch, rows, K, Kp, dst, st);
  if (type == B200_DT_F16) return LaunchSplit<__half>(src, ld, src_mn, o, batch, rows, K, Kp, dst, st);
  return -1;
}

}  // namespace

size_t GemmSplitScratchBytes(int64_t batch, int64_t M, int64_t N, int64_t K, int a_type, int b_type, bool a_mn, bool b_mn,
                             long long lda, long long ldb) {
  const int64_t Kp = (K + BK - 1) / BK * BK;
  // alignment of the caller's pointers is unknown here: size for a copy of a bf16 operand too
  SplitOperand a = PlanOperand(a_type, a_mn, lda, nullptr, batch, M, Kp);
  SplitOperand b = PlanOperand(b_type, b_mn, ldb, nullptr, batch, N, Kp);
  if (a.in_place) a.bytes = 0;
  if (b.in_place) b.bytes = 0;
  return a.bytes + b.bytes;
}

int GemmSplit(const void* A, long long lda, bool a_mn, int a_type, const void* B, long long ldb, bool b_mn, int b_type,
              void* C, int64_t batch, int64_t M, int64_t N, int64_t K, int out_type, cudaStream_t st, void* scratch,
              size_t scratch_bytes, int64_t ldc, int* counter) {
  if (batch <= 0 || M <= 0 || N <= 0) return 0;
  if (ldc <= 0) ldc = N;
  const int out = OutCode(out_type);
  auto ok_type = [](int t) { return t == B200_DT_F32 || t == B200_DT_BF16 || t == B200_DT_F16; };
  if (out < 0 || ldc < N || !ok_type(a_type) || !ok_type(b_type)) return -1;
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX / 8 || batch > 65535 || lda < (a_mn ? M : K) || ldb < (b_mn ? N : K))
    return -1;
  if (K == 0) return cudaMemsetAsync(C, 0, (size_t)batch * M * ldc * (out == 0 ? 4 : 2), st) == cudaSuccess ? 0 : -3;
  const int64_t Kp = (K + BK - 1) / BK * BK;
  const SplitOperand pa = PlanOperand(a_type, a_mn, lda, A, batch, M, Kp);
  const SplitOperand pb = PlanOperand(b_type, b_mn, ldb, B, batch, N, Kp);
  if (pa.bytes + pb.bytes > scratch_bytes || (pa.bytes + pb.bytes && ((uintptr_t)scratch % 256))) return -4;
  // terms (i, j) with i + j <= 2 over the pieces both operands have, smallest first: the f32
  // accumulator then adds the large products last
  Terms tm;
  tm.n = 0;
  for (int sum = 2; sum >= 0; --sum)
    for (int i = sum; i >= 0; --i) {
      const int j = sum - i;
      if (i < pa.pieces && j < pb.pieces) {
        tm.a |= (uint32_t)i << (4 * tm.n);
        tm.b |= (uint32_t)j << (4 * tm.n);
        ++tm.n;
      }
    }
  const void* a_op = A;
  const void* b_op = B;
  long long a_ld = lda, b_ld = ldb;
  bool a_opmn = a_mn, b_opmn = b_mn;
  uint8_t* next = (uint8_t*)scratch;
  if (!pa.in_place) {
    if (int rc = Split(a_type, A, lda, a_mn, pa, batch, M, K, Kp, next, st)) return rc;
    a_op = next;
    a_opmn = pa.dst_mn;
    a_ld = pa.dst_mn ? M : pa.pieces * Kp;
    tm.ka = pa.pieces * Kp;
    next += pa.bytes;
  }
  if (!pb.in_place) {
    if (int rc = Split(b_type, B, ldb, b_mn, pb, batch, N, K, Kp, next, st)) return rc;
    b_op = next;
    b_opmn = pb.dst_mn;
    b_ld = pb.dst_mn ? N : pb.pieces * Kp;
    tm.kb = pb.pieces * Kp;
  }
  // 16-bit results are not split along K here (no f32 workspace): the terms already give every
  // output tile a long K walk
  return RunTc(a_op, a_ld, a_opmn, b_op, b_ld, b_opmn, C, batch, M, N, K, (int64_t)tm.n * Kp, /*bf16*/ 1, out, st,
               out == 0 ? (float*)C : nullptr, ldc, tm, counter);
}

}  // namespace b200k

extern "C" int b200_gemm(const void* A, const void* B, void* C, int64_t batch, int64_t M, int64_t N, int64_t K,
                         int ab_type, int out_type, void* stream) {
  return b200k::Gemm(A, K, B, K, C, batch, M, N, K, ab_type, out_type, (cudaStream_t)stream);
}

extern "C" size_t b200_gemm_split_scratch_bytes(int64_t batch, int64_t M, int64_t N, int64_t K, int a_type, int b_type) {
  if (batch <= 0 || M <= 0 || N <= 0 || K <= 0) return 0;
  return b200k::GemmSplitScratchBytes(batch, M, N, K, a_type, b_type, false, false, K, K);
}

extern "C" int b200_gemm_split(const void* A, int a_type, const void* B, int b_type, void* C, int64_t batch, int64_t M,
                               int64_t N, int64_t K, int out_type, void* scratch, size_t scratch_bytes, void* stream) {
  return b200k::GemmSplit(A, K, false, a_type, B, K, false, b_type, C, batch, M, N, K, out_type, (cudaStream_t)stream,
                          scratch, scratch_bytes, 0);
}
