// attention_bwd_tc.cu — gradient of softmax(scale * Q K^T [causal]) V on the B200 tensor cores:
// dQ, dK, dV from Q, K, V, O, dO and the forward's per-row log2-sum-exp (lse2), bf16 in / out, fp32
// scores, softmax and accumulation.
//
// The reference differentiates attention as plain MPSGraph ops on the full S x S matrices (the
// transpose of the dot_generals of src/jam/ops/linalg.mm and the elementwise softmax VJP).  Here the
// scores are recomputed tile by tile and never leave the SM.
//
// Grid: one CTA per (batch*head, 128-key tile).  The CTA keeps its K and V tiles in shared memory,
// walks the query tiles that can see its keys (all of them, or those at or after the diagonal when
// causal), and accumulates dK and dV in TMEM.  Per query tile (128 queries):
//   S^T  = K Q^T            (M = keys, N = queries, K = head dim)     TMEM cols   0..127
//   dP^T = V dO^T                                                     TMEM cols 128..255
//   P^T  = 2^(S^T * scale * log2 e - lse2[q]),  dS^T = P^T (dP^T - delta[q]) * scale   (CUDA cores)
//   dV  += P^T dO           (A = P^T K-major in smem, B = dO MN-major)                 cols 256..319
//   dK  += dS^T Q           (A = dS^T K-major, B = Q MN-major)                          cols 320..383
//   dQ_t = dS K             (A = the same dS^T tile read MN-major, B = K MN-major)      cols 384..447
// dQ_t is added into an fp32 accumulator in global memory (vector atomics) by a second warpgroup,
// so it overlaps the next tile's score recompute.  delta[q] = sum_d dO[q,d] O[q,d] comes from a
// small preprocessing kernel; a last kernel rounds the dQ accumulator to bf16.
//
//   warp 0     TMA: K, V once; Q, dO tiles (+ lse2, delta slices) through a two-stage ring
//   warp 1     TMEM allocation (512 columns) and the single MMA-issuing thread
//   warps 2-9  P / dS: thread r of warps 2-5 (6-9) owns key row r of the tile (TMEM lane r) for
//              queries 0-63 (64-127) of the step; each half signals its own barrier so the dV / dK
//              products on the first half start while the second is still being computed
//   warps 10-13 dQ readout and atomics: thread r owns query row r
#include <cuda_bf16.h>
#include <mutex>

#include "kernels.h"
#include "tc_common.cuh"
#include "../../../include/b200_kernels.h"

namespace b200k {

static __device__ int g_tc_error_attn_bwd;

namespace {

constexpr int TB = 128;   // keys per CTA tile and queries per step
constexpr int HD = 64;    // head dim

struct BCfg {
  static constexpr int kTile = TB * HD * 2;            // 16 KB: one 128 x 64 bf16 tile
  static constexpr int kKOff = 0;
  static constexpr int kVOff = kKOff + kTile;
  static constexpr int kQOff = kVOff + kTile;         // 2 stages
  static constexpr int kdOOff = kQOff + 2 * kTile;    // 2 stages
  static constexpr int kPOff = kdOOff + 2 * kTile;    // P^T: 128 keys x 128 queries bf16, two 64-query blocks
  static constexpr int kdSOff = kPOff + 2 * kTile;    // dS^T, same layout
  static constexpr int kLseOff = kdSOff + 2 * kTile;  // 2 stages x 128 f32
  static constexpr int kDeltaOff = kLseOff + 2 * TB * 4;
  // dQ staging: per dQ warp two 32-row x 32-column f32 boxes (128-byte swizzled, 4 KB each)
  static constexpr int kdQOff = kDeltaOff + 2 * TB * 4;
  static constexpr int kBarOff = kdQOff + 4 * 2 * 4096;
  static constexpr int kSmem = kBarOff + 256 + 1024;
  static_assert(kdQOff % 1024 == 0, "swizzled boxes need 1024-byte alignment");
};

enum { kKVFull = 0, kQFull = 1, kQEmpty = 3, kSFull = 5, kSFree = 6, kPdSFull = 7 /* 2: per query half */, kPdSFree = 9,
       kdQFull = 10, kdQFree = 11, kAccFull = 12, kNumBars = 13 };
constexpr int kThreads = 14 * 32;   // TMA, MMA, 8 P / dS warps (two query halves), 4 dQ warps

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// f32 box added element-wise into global memory by the TMA unit (an L2 reduction per line)
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];"
               ::"l"(map), "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_group_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// 32 consecutive keys-by-query values of row r, as bf16, into a 128-byte-swizzled K-major tile made
// of two 64-column blocks (column c0 .. c0+31).
__device__ __forceinline__ void store_row32(uint8_t* tile, int r, int c0, const uint32_t (&pk)[16]) {
  uint8_t* rowp = tile + (c0 >> 6) * (TB * 128) + r * 128;
  const int ch0 = (c0 & 63) >> 3;
#pragma unroll
  for (int q = 0; q < 4; ++q)
    *(uint4*)(rowp + (((ch0 + q) ^ (r & 7)) << 4)) = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
}

template <bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1)
attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                const __grid_constant__ CUtensorMap tmdQ,
                const float* __restrict__ lse2, const float* __restrict__ delta, float* __restrict__ dq_acc,
                __nv_bfloat16* __restrict__ dK, __nv_bfloat16* __restrict__ dV, int S, float scale, float scale_log2,
                int dk_t) {
  using C = BCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = (uint64_t*)(smem + C::kBarOff);
  uint32_t* tmem_slot = (uint32_t*)(bars + kNumBars);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_t = S / TB;
  // key-tile-major block order: every (batch, head)'s heaviest key tile (the early keys see the most
  // queries when causal) is dispatched before any lighter one, so the last wave holds short CTAs
  const int n_bh = (int)(gridDim.x / n_t);
  const int kt = (int)(blockIdx.x / n_bh);
  const int bh = (int)(blockIdx.x % n_bh);
  const int k0 = kt * TB;
  const int qt0 = CAUSAL ? kt : 0;
  const int n_it = n_t - qt0;
  const long long row_base = (long long)bh * S;
  int* err = &g_tc_error_attn_bwd;

  if (threadIdx.x == 0) {
    mbar_init(&bars[kKVFull], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[kQFull + i], 1);
      mbar_init(&bars[kQEmpty + i], 1);
    }
    mbar_init(&bars[kSFull], 1);
    mbar_init(&bars[kSFree], 256);
    mbar_init(&bars[kPdSFull + 0], 128);
    mbar_init(&bars[kPdSFull + 1], 128);
    mbar_init(&bars[kPdSFree], 1);
    mbar_init(&bars[kdQFull], 1);
    mbar_init(&bars[kdQFree], 128);
    mbar_init(&bars[kAccFull], 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      prefetch_tmap(&tmdO);
      mbar_arrive_expect_tx(&bars[kKVFull], 2 * C::kTile);
      tma_load_2d_map(&tmK, &bars[kKVFull], smem + C::kKOff, 0, (int)(row_base + k0));
      tma_load_2d_map(&tmV, &bars[kKVFull], smem + C::kVOff, 0, (int)(row_base + k0));
      uint32_t iss = 0, par = 0;
      for (int i = 0; i < n_it; ++i) {
        const int st = i & 1;
        const uint32_t ph = (i >> 1) & 1;
        if (!mbar_wait(&bars[kQEmpty + st], ph ^ 1, kErrTimeoutEmpty, err)) break;
        const int q0 = (qt0 + i) * TB;
        mbar_arrive_expect_tx(&bars[kQFull + st], 2 * C::kTile + 2 * TB * 4);
        tma_load_2d_map(&tmQ, &bars[kQFull + st], smem + C::kQOff + st * C::kTile, 0, (int)(row_base + q0));
        tma_load_2d_map(&tmdO, &bars[kQFull + st], smem + C::kdOOff + st * C::kTile, 0, (int)(row_base + q0));
        bulk_load(smem + C::kLseOff + st * TB * 4, lse2 + row_base + q0, TB * 4, &bars[kQFull + st]);
        bulk_load(smem + C::kDeltaOff + st * TB * 4, delta + row_base + q0, TB * 4, &bars[kQFull + st]);
        iss |= 1u << st;
        par = (par & ~(1u << st)) | (ph << st);
      }
      // never leave with copies in flight
      mbar_wait(&bars[kKVFull], 0, kErrTimeoutOther, err);
      for (int s = 0; s < 2; ++s)
        if (iss & (1u << s)) mbar_wait(&bars[kQFull + s], (par >> s) & 1, kErrTimeoutOther, err);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t id_s = idesc_f16(1, TB, TB);                   // S^T, dP^T: both operands K-major
      const uint32_t id_kv = idesc_f16(1, TB, HD, true);            // dV, dK: B (dO / Q) MN-major
      const uint32_t id_q = idesc_f16(1, TB, HD, true, true);       // dQ: A (dS) and B (K) MN-major
      const uint32_t k_a = smem_u32(smem + C::kKOff), v_a = smem_u32(smem + C::kVOff);
      const uint32_t p_a = smem_u32(smem + C::kPOff), ds_a = smem_u32(smem + C::kdSOff);
      bool ok = mbar_wait(&bars[kKVFull], 0, kErrTimeoutFull, err);
      // S^T = K Q^T and dP^T = V dO^T of step j into TMEM columns 0-255
      auto scores = [&](int j) {
        const int sj = j & 1;
        const uint32_t q_a = smem_u32(smem + C::kQOff + sj * C::kTile), do_a = smem_u32(smem + C::kdOOff + sj * C::kTile);
        if (!mbar_wait(&bars[kQFull + sj], (j >> 1) & 1, kErrTimeoutFull, err)) return false;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          mma_f16_ss(tmem + 0, sw128_desc(k_a + k * 32), sw128_desc(q_a + k * 32), id_s, k != 0);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          mma_f16_ss(tmem + 128, sw128_desc(v_a + k * 32), sw128_desc(do_a + k * 32), id_s, k != 0);
        mma_commit(&bars[kSFull]);
        return true;
      };
      if (ok && n_it > 0) ok = scores(0);
      for (int i = 0; i < n_it && ok; ++i) {
        const int st = i & 1;
        const uint32_t q_a = smem_u32(smem + C::kQOff + st * C::kTile), do_a = smem_u32(smem + C::kdOOff + st * C::kTile);
        // the next step's scores go first: once the P / dS warps have read S^T / dP^T of this step,
        // the tensor core computes the next ones while those warps finish and this step's gradient
        // products below follow
        if (i + 1 < n_it) {
          if (!(ok = mbar_wait(&bars[kSFree], i & 1, kErrTimeoutFull, err))) break;
          if (!(ok = scores(i + 1))) break;
        }
        // dV += P^T dO and dK += dS^T Q: K = 128 queries in steps of 16, issued per 64-query half as
        // soon as that half of P^T / dS^T is in shared memory (the other half is still being written)
        for (int hh = 0; hh < 2 && ok; ++hh) {
          if (!(ok = mbar_wait(&bars[kPdSFull + hh], i & 1, kErrTimeoutFull, err))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const int k = hh * 4 + kk;
            const uint32_t off = hh * (TB * 128) + kk * 32;
            mma_f16_ss(tmem + 256, sw128_desc(p_a + off), sw128_mn_desc_lbo(do_a + k * 2048, 8192), id_kv, (i | k) != 0);
            mma_f16_ss(tmem + 320, sw128_desc(ds_a + off), sw128_mn_desc_lbo(q_a + k * 2048, 8192), id_kv, (i | k) != 0);
          }
        }
        if (!ok) break;
        // dQ_t = dS K: A = dS^T read MN-major (queries contiguous; the two 64-query blocks are the
        // 16 KB-apart MN atoms), K = 128 keys in steps of 16 rows
        if (i > 0 && !(ok = mbar_wait(&bars[kdQFree], (i - 1) & 1, kErrTimeoutFull, err))) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < TB / 16; ++k)
          mma_f16_ss(tmem + 384, sw128_mn_desc_lbo(ds_a + k * 2048, TB * 128), sw128_mn_desc_lbo(k_a + k * 2048, 8192), id_q,
                     k != 0);
        mma_commit(&bars[kPdSFree]);
        mma_commit(&bars[kdQFull]);
        mma_commit(&bars[kQEmpty + st]);
      }
      if (ok) mma_commit(&bars[kAccFull]);
    }
  } else if (warp < 10) {
    // ------------------------------------------------------------------ P / dS (key rows)
    // warps 2-5 take queries 0-63 of each step, warps 6-9 queries 64-127 (same key rows = TMEM lanes)
    const int half = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;           // key row in the tile == TMEM lane
    const int key = k0 + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint8_t* p_tile = smem + C::kPOff;
    uint8_t* ds_tile = smem + C::kdSOff;
    bool ok = true;
    for (int i = 0; i < n_it; ++i) {
      const int st = i & 1;
      const int q0 = (qt0 + i) * TB;
      const float* lse_s = (const float*)(smem + C::kLseOff + st * TB * 4);
      const float* del_s = (const float*)(smem + C::kDeltaOff + st * TB * 4);
      // the lse2 / delta slices arrive with the Q / dO tiles of this stage
      if (!(ok = mbar_wait_warp(&bars[kQFull + st], (i >> 1) & 1, kErrTimeoutAcc, err))) break;
      if (!(ok = mbar_wait_warp(&bars[kSFull], i & 1, kErrTimeoutAcc, err))) break;
      tc_fence_after();
      const bool diag = CAUSAL && q0 == k0;
#pragma unroll 1
      for (int c = half * 64; c < half * 64 + 64; c += 32) {
        uint32_t sv[32], dv[32];
        tmem_ld16(tmem + lane_off + c, *reinterpret_cast<uint32_t(*)[16]>(sv));
        tmem_ld16(tmem + lane_off + c + 16, *reinterpret_cast<uint32_t(*)[16]>(sv + 16));
        tmem_ld16(tmem + lane_off + 128 + c, *reinterpret_cast<uint32_t(*)[16]>(dv));
        tmem_ld16(tmem + lane_off + 128 + c + 16, *reinterpret_cast<uint32_t(*)[16]>(dv + 16));
        tmem_wait_ld();
        if (c == half * 64 + 32) {                // last TMEM read of this step: S^T / dP^T may be
          tc_fence_before();                      // recomputed for the next step
          mbar_arrive(&bars[kSFree]);
        }
        uint32_t pp[16], pd[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float p0 = ex2f(fmaf(__uint_as_float(sv[e]), scale_log2, -lse_s[c + e]));
          float p1 = ex2f(fmaf(__uint_as_float(sv[e + 1]), scale_log2, -lse_s[c + e + 1]));
          if (diag) {                             // keys after the query do not contribute
            if (key > q0 + c + e) p0 = 0.f;
            if (key > q0 + c + e + 1) p1 = 0.f;
          }
          const float d0 = p0 * (__uint_as_float(dv[e]) - del_s[c + e]) * scale;
          const float d1 = p1 * (__uint_as_float(dv[e + 1]) - del_s[c + e + 1]) * scale;
          pp[e >> 1] = pack_bf16x2(p0, p1);
          pd[e >> 1] = pack_bf16x2(d0, d1);
        }
        // the previous step's P / dS may still be read by its dV / dK / dQ products
        if (c == half * 64 && i > 0 && !(ok = mbar_wait_warp(&bars[kPdSFree], (i - 1) & 1, kErrTimeoutAcc, err))) break;
        store_row32(p_tile, r, c, pp);
        store_row32(ds_tile, r, c, pd);
      }
      if (!ok) break;
      fence_async_shared();
      mbar_arrive(&bars[kPdSFull + half]);
    }
    // dV and dK rows of this key tile
    if (ok && mbar_wait_warp(&bars[kAccFull], 0, kErrTimeoutAcc, err)) {
      tc_fence_after();
      for (int w = half; w < half + 1; ++w) {  // half 0 writes dV, half 1 dK
        __nv_bfloat16* out = (w == 0 ? dV : dK) + (row_base + key) * HD;
        const uint32_t col = tmem + lane_off + 256 + w * 64;
        if (w == 1 && dk_t) {
          // dK as [B*H, D, S] (the layout a dot_general(Q, dS) result has): for each d the warp's 32
          // consecutive keys form one 64-byte store
          __nv_bfloat16* outt = dK + (long long)bh * HD * S + key;
#pragma unroll 1
          for (int c = 0; c < HD; c += 16) {
            uint32_t v[16];
            tmem_ld16(col + c, v);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) outt[(long long)(c + e) * S] = __float2bfloat16_rn(__uint_as_float(v[e]));
          }
          continue;
        }
#pragma unroll
        for (int c = 0; c < HD; c += 16) {
          uint32_t v[16];
          tmem_ld16(col + c, v);
          tmem_wait_ld();
          uint4 w0 = make_uint4(pack_bf16x2(__uint_as_float(v[0]), __uint_as_float(v[1])),
                                pack_bf16x2(__uint_as_float(v[2]), __uint_as_float(v[3])),
                                pack_bf16x2(__uint_as_float(v[4]), __uint_as_float(v[5])),
                                pack_bf16x2(__uint_as_float(v[6]), __uint_as_float(v[7])));
          uint4 w1 = make_uint4(pack_bf16x2(__uint_as_float(v[8]), __uint_as_float(v[9])),
                                pack_bf16x2(__uint_as_float(v[10]), __uint_as_float(v[11])),
                                pack_bf16x2(__uint_as_float(v[12]), __uint_as_float(v[13])),
                                pack_bf16x2(__uint_as_float(v[14]), __uint_as_float(v[15])));
          *(uint4*)(out + c) = w0;
          *(uint4*)(out + c + 8) = w1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ dQ readout (query rows)
    // each warp's 32 query rows leave as two 32 x 32 f32 boxes added into dq_acc by TMA reductions
    // (whole 128-byte lines per L2 operation instead of one 16-byte atomic per row and chunk)
    const int quarter = warp & 3;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint8_t* boxes = smem + C::kdQOff + quarter * 8192;
    for (int i = 0; i < n_it; ++i) {
      if (!mbar_wait_warp(&bars[kdQFull], i & 1, kErrTimeoutAcc, err)) break;
      tc_fence_after();
      const int row0 = (int)(row_base + (long long)(qt0 + i) * TB + quarter * 32);
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        uint32_t v[32];
        tmem_ld16(tmem + lane_off + 384 + h * 32, *reinterpret_cast<uint32_t(*)[16]>(v));
        tmem_ld16(tmem + lane_off + 384 + h * 32 + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
        tmem_wait_ld();
        if (h == 1) {                             // both columns read: the MMA may overwrite dQ_t
          tc_fence_before();
          mbar_arrive(&bars[kdQFree]);
        }
        uint8_t* box = boxes + h * 4096;
        if (lane == 0) bulk_wait_group_read0();   // this box's previous reduction has read it
        __syncwarp();
#pragma unroll
        for (int q = 0; q < 8; ++q)
          *(uint4*)(box + lane * 128 + ((q ^ (lane & 7)) << 4)) = make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        fence_async_shared();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_2d(&tmdQ, box, h * 32, row0);
          bulk_commit_group();
        }
      }
    }
    if (lane == 0) bulk_wait_group0();            // reductions complete before the CTA exits
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// delta = rowsum(dO * O): eight threads per 64-element row, one 16-byte load of each operand per
// thread, a three-step shuffle; a warp covers four rows per step (512 contiguous bytes per load)
__global__ void __launch_bounds__(256) attn_bwd_delta_kernel(const __nv_bfloat16* __restrict__ O,
                                                             const __nv_bfloat16* __restrict__ dO, float* __restrict__ delta,
                                                             long long rows) {
  const int sub = threadIdx.x & 7, lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * 8;
  // warp-uniform loop over groups of four rows; a row past the end contributes nothing
  for (long long r4 = ((long long)blockIdx.x * 256 + threadIdx.x) >> 5; r4 * 4 < rows; r4 += warps) {
    const long long row = r4 * 4 + (lane >> 3);
    float s = 0.f;
    if (row < rows) {
      const uint4 o = ((const uint4*)(O + row * HD))[sub];
      const uint4 g = ((const uint4*)(dO + row * HD))[sub];
      const __nv_bfloat162* o2 = (const __nv_bfloat162*)&o;
      const __nv_bfloat162* g2 = (const __nv_bfloat162*)&g;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 a = __bfloat1622float2(o2[e]), b = __bfloat1622float2(g2[e]);
        s = fmaf(a.x, b.x, s);
        s = fmaf(a.y, b.y, s);
      }
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    if (sub == 0 && row < rows) delta[row] = s;
  }
}

__global__ void __launch_bounds__(256) f32_to_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                                          long long n4) {
  for (long long i = (long long)blockIdx.x * 256 + threadIdx.x; i < n4; i += (long long)gridDim.x * 256) {
    const float4 v = ((const float4*)x)[i];
    ((uint2*)y)[i] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

}  // namespace

EncodeTiledFn GetEncodeTiled();

// [rows, 64] bf16, 128 x 64 boxes, 128-byte swizzle.
// dq_acc rows (64 f32) as 32 x 32 boxes, 128-byte swizzled, for the TMA reductions
static bool MapRowsF32(CUtensorMap* map, const void* ptr, uint64_t rows) {
  EncodeTiledFn enc = GetEncodeTiled();
  if (!enc) return false;
  cuuint64_t dims[2] = {HD, rows};
  cuuint64_t strides[1] = {HD * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(ptr), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool MapRows64(CUtensorMap* map, const void* ptr, uint64_t rows) {
  EncodeTiledFn enc = GetEncodeTiled();
  if (!enc) return false;
  cuuint64_t dims[2] = {HD, rows};
  cuuint64_t strides[1] = {HD * 2};
  cuuint32_t box[2] = {64, TB};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool AttentionBwdShapeOk(int B, int H, int S, int D) {
  if (!(B > 0 && H > 0 && D == HD && S > 0 && S % TB == 0)) return false;
  long long bh = 0, rows = 0;   // overflow-checked: huge dimensions must not wrap to a small product
  return !__builtin_mul_overflow((long long)B, (long long)H, &bh) && !__builtin_mul_overflow(bh, (long long)S, &rows) &&
         rows <= INT32_MAX;
}

// Scratch: dq_acc (B*H*S*D f32) and delta (B*H*S f32), caller-owned.  Allocates nothing.
// dk_t: dK is written as [B, H, D, S] instead of [B, H, S, D].
int AttentionBwd(const void* q, const void* k, const void* v, const void* o, const void* dout, const float* lse2,
                 void* dq, void* dk, void* dv, float* dq_acc, float* delta, int B, int H, int S, int D, int causal,
                 float scale, cudaStream_t st, int dk_t = 0) {
  if (!AttentionBwdShapeOk(B, H, S, D)) return -1;
  if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)o | (uintptr_t)dout | (uintptr_t)dq | (uintptr_t)dk |
       (uintptr_t)dv | (uintptr_t)lse2 | (uintptr_t)dq_acc | (uintptr_t)delta) % 16)
    return -1;
  using C = BCfg;
  static std::once_flag once[8][2];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 7][causal ? 1 : 0], [causal] {
    if (causal) cudaFuncSetAttribute(attn_bwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    else cudaFuncSetAttribute(attn_bwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  });
  const long long rows = (long long)B * H * S;
  CUtensorMap mq, mk, mv, mdo;
  CUtensorMap mdq;
  if (!MapRows64(&mq, q, rows) || !MapRows64(&mk, k, rows) || !MapRows64(&mv, v, rows) || !MapRows64(&mdo, dout, rows) ||
      !MapRowsF32(&mdq, dq_acc, rows))
    return -2;
  if (cudaMemsetAsync(dq_acc, 0, (size_t)rows * HD * 4, st) != cudaSuccess) return -3;
  attn_bwd_delta_kernel<<<(unsigned)std::min<long long>((rows + 31) / 32, 148 * 8), 256, 0, st>>>(
      (const __nv_bfloat16*)o, (const __nv_bfloat16*)dout, delta, rows);
  CountLaunches();
  const float scale_log2 = scale * 1.4426950408889634f;
  dim3 grid((unsigned)(B * H * (S / TB)));
  if (causal)
    attn_bwd_kernel<true><<<grid, kThreads, C::kSmem, st>>>(mq, mk, mv, mdo, mdq, lse2, delta, dq_acc, (__nv_bfloat16*)dk,
                                                        (__nv_bfloat16*)dv, S, scale, scale_log2, dk_t);
  else
    attn_bwd_kernel<false><<<grid, kThreads, C::kSmem, st>>>(mq, mk, mv, mdo, mdq, lse2, delta, dq_acc, (__nv_bfloat16*)dk,
                                                         (__nv_bfloat16*)dv, S, scale, scale_log2, dk_t);
  CountLaunches();
  // dq null: the caller reads dQ (rounding it itself) from the f32 accumulator
  const long long n4 = rows * HD / 4;
  if (dq) {
    f32_to_bf16_kernel<<<(unsigned)std::min<long long>((n4 + 255) / 256, 148 * 8), 256, 0, st>>>(dq_acc, (__nv_bfloat16*)dq, n4);
    CountLaunches();
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int TakeAttnBwdError() {
  int v = 0, z = 0;
  cudaMemcpyFromSymbol(&v, g_tc_error_attn_bwd, sizeof(int));
  if (v) cudaMemcpyToSymbol(g_tc_error_attn_bwd, &z, sizeof(int));
  return v;
}

}  // namespace b200k

extern "C" int b200_attention_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
                                  const float* lse2, void* dq, void* dk, void* dv, float* dq_acc, float* delta, int B,
                                  int H, int S, int D, int causal, float scale, void* stream) {
  if (B == 0 || H == 0 || S == 0) return 0;
  return b200k::AttentionBwd(q, k, v, o, dout, lse2, dq, dk, dv, dq_acc, delta, B, H, S, D, causal, scale,
                             (cudaStream_t)stream);
}
