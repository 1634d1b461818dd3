// tied_ce.cu — B200 (sm_100a) fused tied LM-head cross-entropy.
//
// The reference computes, on CuPy/NumPy (NimbleML/kernels/fused_tied_crossentropy.py:8-48,
// NimbleML/kernels/fused_crossentropy.py:14-50):
//   forward : S = h E^T (N x V, materialised); m = rowmax S; s = sum exp(S - m);
//             lse = m + log s; loss = mean_i (lse_i - S_i,y_i)
//   backward: G = (exp(S - m) / s - onehot(y)) * grad_scale / N
//             dh = G E ; dE = G^T h
// Here nothing N x V is ever stored:
//   forward : one persistent tcgen05 GEMM over (token block x vocab tile)
//             tiles whose epilogue reduces each TMEM accumulator row to a
//             (max, sum-exp) pair and gathers the target logit; a row reduce
//             merges the per-tile pairs; a combine kernel merges vocab shards
//             and forms lse and the loss.
//   backward: per vocab slab of the shard, the same GEMM recomputes the
//             logits and its epilogue writes G for that slab only; two more
//             tcgen05 GEMMs give dE rows of the slab (complete) and add the
//             slab's share of dh, reading G, h and E in place (MN-major
//             operands where the contraction runs along their rows).
// All GEMMs compute C[M x N] = A[M x K] . B[N x K]^T with operands staged by
// TMA (128-byte swizzle) into a shared-memory ring and fp32 accumulators
// double-buffered in TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "nimbleml_tied_ce.h"
#include "common.cuh"
#include "sm100_ptx.cuh"

namespace nimble {

// ------------------------------------------------------------------ tiling
constexpr int kBM = 128;          // accumulator rows per tile (TMEM lanes)
constexpr int kBN = 256;          // accumulator columns per tile
constexpr int kBKBytes = 128;     // one 128-byte swizzle row of K per stage
constexpr int kStages = 4;        // shared-memory ring depth
constexpr int kABytes = kBM * kBKBytes;  // 16 KiB
constexpr int kBBytes = kBN * kBKBytes;  // 32 KiB
constexpr int kEpiWarps = 8;      // two per TMEM lane quarter, each on half the columns
constexpr int kColHalves = kEpiWarps / 4;
constexpr int kThreads = 64 + 32 * kEpiWarps;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kTmemCols = 2 * kBN;  // two accumulators
// Staging for the G tile stores: 32 KiB shared by the epilogue warps, i.e.
// two 32 x 32 buffers per warp for 16-bit G, one for fp32 G.
constexpr int kStoreBytes = 32768;
constexpr int kSmemBytes = kStages * (kABytes + kBBytes) + kStoreBytes + 1024 /*align*/ + 256 /*barriers*/;
// CTA-pair mode (cta_group::2): each CTA holds 128 rows of A and 128 of the
// 256 B rows per stage (32 KiB), so the ring is 6 stages deep.
constexpr int kStagesPair = 6;
// Wide single-CTA tiles: 32 KiB of A + 32 KiB of B per stage.
constexpr int kStagesWide = 3;
constexpr int kSmemBytesPair = kStagesPair * (kABytes + kBBytes / 2) + kStoreBytes + 1024 + 256;
constexpr float kLog2e = 1.4426950408889634f;

enum Epi : int { EPI_CE_FWD = 0, EPI_CE_GRAD = 1, EPI_STORE = 2 };

struct EpiParams {
  // Shared by the cross-entropy epilogues.
  const int64_t* labels;   // [M] global class ids
  int64_t col_origin;      // global class id of B row 0
  int64_t ignore_index;
  // EPI_CE_FWD
  float2* part;            // [n_tiles][M] per-tile (max, sum-exp)
  float* tgt;              // [M] target logit, written by the owning tile
  // EPI_CE_GRAD
  const float* lse;        // [M]
  void* g;                 // [M][ldg]    G * gscale, compute dtype
  int64_t ldg;
  float gscale;
  // EPI_STORE: out = alpha * (acc + src) (+ out if accum_out)
  void* out;
  int64_t ld_out;
  int out_dtype;
  const float* src;
  int64_t ld_src;
  const float* alpha_num;  // device scalar or null (1)
  const float* alpha_den;  // device scalar or null (1); alpha = 0 when *den == 0
  float alpha_mult;
  int accum_out;
  int* status;
};

template <typename T> struct ElemInfo;
template <> struct ElemInfo<__half> {
  static constexpr uint32_t kFmt = 0; static constexpr bool kTF32 = false;
};
template <> struct ElemInfo<__nv_bfloat16> {
  static constexpr uint32_t kFmt = 1; static constexpr bool kTF32 = false;
};
template <> struct ElemInfo<float> {
  static constexpr uint32_t kFmt = 2; static constexpr bool kTF32 = true;
};

__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int group_m, int& mb, int& nb) {
  // Groups of `group_m` token blocks sweep the vocab tiles together so the
  // concurrently resident tiles share A and B blocks in L2.
  const int per_group = group_m * n_tiles;
  const int g = t / per_group;
  const int first_m = g * group_m;
  const int gsz = min(group_m, m_tiles - first_m);
  const int r = t - g * per_group;
  mb = first_m + r % gsz;
  nb = r / gsz;
}

template <typename T>
__device__ __forceinline__ T to_elem(float x);
template <> __device__ __forceinline__ __half to_elem<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 to_elem<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <> __device__ __forceinline__ float to_elem<float>(float x) { return ptx::round_tf32(x); }

__device__ __forceinline__ uint32_t pack2(__half a, __half b) {
  return static_cast<uint32_t>(__half_as_ushort(a)) | (static_cast<uint32_t>(__half_as_ushort(b)) << 16);
}
__device__ __forceinline__ uint32_t pack2(__nv_bfloat16 a, __nv_bfloat16 b) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(a)) |
         (static_cast<uint32_t>(__bfloat16_as_ushort(b)) << 16);
}

__device__ __forceinline__ float load_out_elem(const void* p, int64_t i, int dt) {
  if (dt == NIMBLE_DTYPE_F32) return static_cast<const float*>(p)[i];
  if (dt == NIMBLE_DTYPE_F16) return __half2float(static_cast<const __half*>(p)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}
__device__ __forceinline__ void store_out_elem(void* p, int64_t i, int dt, float v) {
  if (dt == NIMBLE_DTYPE_F32) static_cast<float*>(p)[i] = v;
  else if (dt == NIMBLE_DTYPE_F16) static_cast<__half*>(p)[i] = __float2half_rn(v);
  else static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

// ------------------------------------------------------------- the GEMM
// Persistent, warp-specialised: warp 0 lane 0 issues TMA loads into a
// shared-memory ring, warp 1 lane 0 issues tcgen05.mma into TMEM, and warps
// 2-9 run the epilogue (two warps per TMEM lane quarter, each on half of the
// 256 columns, one thread per accumulator row). With 128 x 256 tiles the two
// TMEM accumulators alternate, so the epilogue of tile i overlaps the MMAs of
// tile i+1. kAMN / kBMN select an
// MN-major A / B operand (the tensor map's inner dimension is then M / N and
// the tile arrives as 128-byte-wide MN chunks of K rows).
//
// kCG = 2 runs CTA pairs (clusters of 2): the pair computes a 256 x 256 tile
// with tcgen05.mma.cta_group::2 issued by the even CTA; each CTA loads its own
// 128 A rows and 128 of the B rows, its TMEM holds its 128 accumulator rows,
// and its epilogue warps write them. Loads are never multicast.
//
// kWide (one CTA) computes a 256 x 256 tile as two M=128 MMAs per K step that
// share the B tile, accumulating into all 512 TMEM columns: a third fewer
// operand bytes per FLOP than 128 x 256 tiles, but the epilogue of a tile no
// longer overlaps the next tile's MMAs.
template <typename T, int EPI, bool kAMN, bool kBMN, int kCG, bool kWide = false>
__global__ void __launch_bounds__(kThreads, 1)
tc_gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const __grid_constant__ CUtensorMap tmC, int M, int N, int K, int group_m, EpiParams ep) {
  static_assert(!(kWide && kCG == 2), "wide tiles are single-CTA");
  constexpr int kMB = kWide ? 2 : 1;                      // 128-row M blocks per CTA
  constexpr int kS = kCG == 2 ? kStagesPair : (kWide ? kStagesWide : kStages);  // ring depth
  constexpr int kBRows = kBN / kCG;                       // B rows loaded per CTA
  constexpr int kBBytesCta = kBRows * kBKBytes;
  constexpr int kABytesCta = kABytes * kMB;
  constexpr int kTileM = kBM * kCG * kMB;                 // accumulator rows per tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kS * kABytesCta;
  uint8_t* sStore = sB + kS * kBBytesCta;  // 1024-aligned: stage sizes are multiples of 1 KiB
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sStore + kStoreBytes);
  uint64_t* empty_bar = full_bar + kS;
  uint64_t* tfull_bar = empty_bar + kS;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  constexpr int kElem = sizeof(T);
  constexpr int kBK = kBKBytes / kElem;           // K elements per stage
  constexpr int kUK = 32 / kElem;                 // K elements per MMA (32 bytes)
  constexpr int kKSteps = kBK / kUK;              // MMAs per stage
  constexpr bool kTF32 = ElemInfo<T>::kTF32;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = (M + kTileM - 1) / kTileM;
  const int n_tiles = (N + kBN - 1) / kBN;
  const int tiles = m_tiles * n_tiles;
  const int k_blocks = (K + kBK - 1) / kBK;
  const uint32_t rank = kCG == 2 ? ptx::cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int unit0 = blockIdx.x / kCG;       // this CTA's first tile
  const int units = gridDim.x / kCG;        // tile stride

  if (threadIdx.x == 0) {
    for (int s = 0; s < kS; ++s) {
      ptx::mbar_init(&full_bar[s], 1);
      ptx::mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&tfull_bar[a], 1);
      ptx::mbar_init(&tempty_bar[a], kEpiWarps * kCG);
    }
    ptx::mbar_init(drain_bar, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::fence_proxy_async_smem();
  }
  if (warp == 1) ptx::tmem_alloc_cg<kCG>(tmem_slot, kTmemCols);
  ptx::tc_fence_before();
  __syncthreads();
  if constexpr (kCG == 2) ptx::cluster_sync();  // peer barriers initialised
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      ptx::prefetch_tmap(&tmA);
      ptx::prefetch_tmap(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;  // bit s: stage s has a load outstanding-or-done
      bool ok = true;
      auto load = [&](void* dst, const CUtensorMap* m, int stg, int x, int y) {
        if constexpr (kCG == 2)
          ptx::tma_load_2d_pair(dst, m, ptx::mapa_shared(&full_bar[stg], 0), x, y);
        else
          ptx::tma_load_2d(dst, m, &full_bar[stg], x, y);
      };
      for (int t = unit0; t < tiles && ok; t += units) {
        int mb, nb;
        tile_coords(t, m_tiles, n_tiles, group_m, mb, nb);
        const int a_row0 = mb * kTileM + static_cast<int>(rank) * kBM;
        const int b_row0 = nb * kBN + static_cast<int>(rank) * kBRows;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!ptx::mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag)) { ok = false; break; }
          // The even CTA's full barrier counts both CTAs' bytes.
          if (leader) ptx::mbar_arrive_expect_tx(&full_bar[stage], kCG * (kABytesCta + kBBytesCta));
          if constexpr (kAMN) {
#pragma unroll
            for (int j = 0; j < kMB * kBM / kBK; ++j)
              load(sA + stage * kABytesCta + j * kBK * 128, &tmA, stage, a_row0 + j * kBK, kb * kBK);
          } else {
#pragma unroll
            for (int q = 0; q < kMB; ++q)
              load(sA + stage * kABytesCta + q * kABytes, &tmA, stage, kb * kBK, a_row0 + q * kBM);
          }
          if constexpr (kBMN) {
#pragma unroll
            for (int j = 0; j < kBRows / kBK; ++j)
              load(sB + stage * kBBytesCta + j * kBK * 128, &tmB, stage, b_row0 + j * kBK, kb * kBK);
          } else {
            load(sB + stage * kBBytesCta, &tmB, stage, kb * kBK, b_row0);
          }
          issued |= 1u << stage;
          if (++stage == kS) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok && leader) {
        // Let every load already issued land before the CTA can exit: the
        // most recent phase of each stage is `phase` for stages below the
        // cursor and `phase ^ 1` at or above it.
        for (int s = 0; s < kS; ++s) {
          if (!(issued & (1u << s))) continue;
          const uint32_t par = (s < stage) ? phase : (phase ^ 1);
          const uint64_t t0 = ptx::globaltimer_ns();
          while (!ptx::mbar_try_wait(&full_bar[s], par) && ptx::globaltimer_ns() - t0 < ptx::kWaitLimitNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------ MMA issuer
      // M of one instruction: 128 per CTA, 256 for a CTA pair (never the wide tile's 256).
      constexpr uint32_t idesc = ptx::idesc_f32acc(ElemInfo<T>::kFmt, kBM * kCG, kBN, kAMN, kBMN);
      // Start-address step (16-byte units) per MMA along K: 32 bytes inside a
      // K-major swizzle row, or kUK rows of 128 bytes for an MN-major tile.
      constexpr uint64_t kAStep = kAMN ? kUK * 128 / 16 : 2;
      constexpr uint64_t kBStep = kBMN ? kUK * 128 / 16 : 2;
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int t = unit0; t < tiles && ok; t += units, ++it) {
        const int acc = kWide ? 0 : (it & 1);
        const uint32_t aphase = kWide ? (it & 1) : ((it >> 1) & 1);
        if (!ptx::mbar_wait(&tempty_bar[acc], aphase ^ 1, abort_flag)) { ok = false; break; }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kBN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!ptx::mbar_wait(&full_bar[stage], phase, abort_flag)) { ok = false; break; }
          ptx::tc_fence_after();
          const uint32_t a_addr = ptx::smem_u32(sA + stage * kABytesCta);
          const uint32_t b_addr = ptx::smem_u32(sB + stage * kBBytesCta);
          const uint64_t adesc = kAMN ? ptx::sdesc_mn_sw128(a_addr, kBK * 128, kTF32) : ptx::sdesc_k_sw128(a_addr);
          const uint64_t bdesc = kBMN ? ptx::sdesc_mn_sw128(b_addr, kBK * 128, kTF32) : ptx::sdesc_k_sw128(b_addr);
#pragma unroll
          for (int k = 0; k < kKSteps; ++k) {
            if constexpr (kCG == 2)
              ptx::umma_pair<kTF32>(d_tmem, adesc + kAStep * k, bdesc + kBStep * k, idesc, (kb | k) != 0 ? 1u : 0u);
            else
              ptx::umma<kTF32>(d_tmem, adesc + kAStep * k, bdesc + kBStep * k, idesc, (kb | k) != 0 ? 1u : 0u);
            if constexpr (kWide) {
              // Second M block: A rows 128..255 sit 16 KiB further in the stage.
              ptx::umma<kTF32>(d_tmem + kBN, adesc + (kABytes >> 4) + kAStep * k, bdesc + kBStep * k, idesc,
                               (kb | k) != 0 ? 1u : 0u);
            }
          }
          // Frees this stage in both CTAs once the MMAs have read it.
          if constexpr (kCG == 2) ptx::umma_commit_pair(&empty_bar[stage], 0x3);
          else ptx::umma_commit(&empty_bar[stage]);
          if (++stage == kS) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        if constexpr (kCG == 2) ptx::umma_commit_pair(&tfull_bar[acc], 0x3);
        else ptx::umma_commit(&tfull_bar[acc]);
      }
      if (!ok) {
        // Drain: wait until every MMA issued so far has finished.
        if constexpr (kCG == 2) ptx::umma_commit_pair(drain_bar, 0x1);
        else ptx::umma_commit(drain_bar);
        const uint64_t t0 = ptx::globaltimer_ns();
        while (!ptx::mbar_try_wait(drain_bar, 0) && ptx::globaltimer_ns() - t0 < ptx::kWaitLimitNs) {
        }
      }
    }
  } else {
    // ---------------------------------------------------- epilogue
    const int wq = warp & 3;  // TMEM lane quarter this warp may access
    const int row_t = wq * 32 + lane;
    const int ew = warp - 2;                        // epilogue warp index
    const int ch = ew / 4;                          // which half of the 256 columns
    constexpr int kChunks32 = kBN / 32 / kColHalves;  // 32-column chunks per warp
    const int c_begin = ch * kChunks32, c_end = c_begin + kChunks32;
    float alpha = 1.0f;
    if constexpr (EPI == EPI_STORE) {
      const float num = ep.alpha_num ? *ep.alpha_num : 1.0f;
      const float den = ep.alpha_den ? *ep.alpha_den : 1.0f;
      alpha = (den != 0.0f) ? num / den * ep.alpha_mult : 0.0f;
    }
    // TMEM of an accumulator is handed back to the MMA issuer (even CTA).
    auto release = [&](int acc) {
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (kCG == 2) ptx::mbar_arrive_cluster(ptx::mapa_shared(&tempty_bar[acc], 0));
        else ptx::mbar_arrive(&tempty_bar[acc]);
      }
    };
    int it = 0;
    int store_seq = 0;  // G staging stores issued by this warp
    for (int t = unit0; t < tiles; t += units, ++it) {
      int mb, nb;
      tile_coords(t, m_tiles, n_tiles, group_m, mb, nb);
      const int acc = kWide ? 0 : (it & 1);
      const uint32_t aphase = kWide ? (it & 1) : ((it >> 1) & 1);
      bool ok = ptx::mbar_wait(&tfull_bar[acc], aphase, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      ptx::tc_fence_after();
#pragma unroll 1
      for (int rb = 0; rb < kMB; ++rb) {
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(wq * 32) << 16) + (acc + rb) * kBN;
      const int64_t row =
          static_cast<int64_t>(mb) * kTileM + static_cast<int64_t>(rank) * kBM + rb * kBM + row_t;
      const bool row_ok = row < M;
      const int ncols = min(kBN, N - nb * kBN);
      const int64_t col0_tile = static_cast<int64_t>(nb) * kBN;

      if constexpr (EPI == EPI_CE_FWD) {
        const int64_t lab = row_ok ? ep.labels[row] : INT64_MIN;
        const int64_t rel = (lab == INT64_MIN) ? -1 : lab - ep.col_origin - col0_tile;
        const int tcol = (rel >= 0 && rel < ncols) ? static_cast<int>(rel) : -1;
        float mrun = -INFINITY, srun = 0.0f, tval = 0.0f;
#pragma unroll 1
        for (int c = c_begin; c < c_end; ++c) {
          if (c * 32 >= ncols) break;
          uint32_t r[32];
          __syncwarp();
          ptx::tmem_ld_32cols(tbase + c * 32, r);
          ptx::tmem_wait_ld();
          ptx::tmem_fence_regs(r);
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          const int nv = ncols - c * 32;
          if (nv < 32) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j >= nv) v[j] = -INFINITY;
          }
          float cm = v[0];
#pragma unroll
          for (int j = 1; j < 32; ++j) cm = fmaxf(cm, v[j]);
          const float mnew = fmaxf(mrun, cm);
          const float ml2 = mnew * kLog2e;
          float s0 = 0.f, s1 = 0.f;
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            s0 += ptx::ex2(fmaf(v[j], kLog2e, -ml2));
            s1 += ptx::ex2(fmaf(v[j + 1], kLog2e, -ml2));
          }
          srun = srun * ptx::ex2((mrun - mnew) * kLog2e) + (s0 + s1);
          mrun = mnew;
          const int jt = tcol - c * 32;
          if (static_cast<unsigned>(jt) < 32u) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j == jt) tval = v[j];
          }
        }
        if (row_ok) {
          ep.part[(static_cast<int64_t>(nb) * kColHalves + ch) * M + row] = make_float2(mrun, srun);
          // Only the warp whose column half holds the label writes the target.
          if (tcol >= c_begin * 32 && tcol < c_end * 32) ep.tgt[row] = tval;
        }
      } else if constexpr (EPI == EPI_CE_GRAD) {
        const int64_t lab = row_ok ? ep.labels[row] : ep.ignore_index;
        const bool live = row_ok && lab != ep.ignore_index;
        const int64_t rel = live ? lab - ep.col_origin - col0_tile : -1;
        const int tcol = (rel >= 0 && rel < ncols) ? static_cast<int>(rel) : -1;
        const float lse_l2 = live ? ep.lse[row] * kLog2e : 0.0f;
        const float gs = live ? ep.gscale : 0.0f;
        // The warp's 32 rows x 32 columns of G go through a swizzled staging
        // buffer and one TMA store (rows >= M / columns >= N are clipped by
        // the tensor map). Row bytes: 64 (16-bit, 64-byte swizzle) or 128
        // (fp32, 128-byte swizzle).
        constexpr int kRowBytes = 32 * kElem;
        constexpr int kChunks = kRowBytes / 16;
        const int swz = kElem == 2 ? ((lane >> 1) & 3) : (lane & 7);
        constexpr int kBufBytes = 32 * kRowBytes;
        constexpr int kBufs = kStoreBytes / (kEpiWarps * kBufBytes) >= 2 ? 2 : 1;
        static_assert(kEpiWarps * kBufs * kBufBytes <= kStoreBytes, "G staging exceeds its shared memory");
        uint8_t* wbuf = sStore + ew * kBufs * kBufBytes;
        const int store_row0 = mb * kTileM + static_cast<int>(rank) * kBM + rb * kBM + wq * 32;
#pragma unroll 1
        for (int c = c_begin; c < c_end; ++c) {
          if (c * 32 >= ncols) break;
          uint32_t r[32];
          __syncwarp();
          ptx::tmem_ld_32cols(tbase + c * 32, r);
          ptx::tmem_wait_ld();
          ptx::tmem_fence_regs(r);
          const int jt = tcol - c * 32;
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float p = ptx::ex2(fmaf(__uint_as_float(r[j]), kLog2e, -lse_l2));
            if (j == jt) p -= 1.0f;
            v[j] = p * gs;
          }
          uint8_t* buf = wbuf + (store_seq % kBufs) * kBufBytes;
          if (store_seq >= kBufs && lane == 0) ptx::bulk_wait_read<kBufs - 1>();  // buffer's last store has read it
          __syncwarp();
          alignas(16) T vals[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) vals[j] = to_elem<T>(v[j]);
#pragma unroll
          for (int q = 0; q < kChunks; ++q)
            *reinterpret_cast<uint4*>(buf + lane * kRowBytes + ((q ^ swz) * 16)) =
                *reinterpret_cast<const uint4*>(&vals[q * (16 / kElem)]);
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            ptx::tma_store_2d(&tmC, buf, static_cast<int>(col0_tile) + c * 32, store_row0);
            ptx::bulk_commit();
          }
          ++store_seq;
        }
      } else {  // EPI_STORE
#pragma unroll 1
        for (int c = c_begin; c < c_end; ++c) {
          if (c * 32 >= ncols) break;
          uint32_t r[32];
          __syncwarp();
          ptx::tmem_ld_32cols(tbase + c * 32, r);
          ptx::tmem_wait_ld();
          ptx::tmem_fence_regs(r);
          if (!row_ok) continue;
          const int64_t col = col0_tile + c * 32;
          const int nv = min(32, ncols - c * 32);
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          if (nv == 32) {
            if (ep.src) {
              const float4* s4 = reinterpret_cast<const float4*>(ep.src + row * ep.ld_src + col);
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const float4 a = s4[q];
                v[4 * q] += a.x; v[4 * q + 1] += a.y; v[4 * q + 2] += a.z; v[4 * q + 3] += a.w;
              }
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] *= alpha;
            if (ep.out_dtype == NIMBLE_DTYPE_F32) {
              float4* o4 = reinterpret_cast<float4*>(static_cast<float*>(ep.out) + row * ep.ld_out + col);
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                float4 o = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                if (ep.accum_out) {
                  const float4 a = o4[q];
                  o.x += a.x; o.y += a.y; o.z += a.z; o.w += a.w;
                }
                o4[q] = o;
              }
            } else {
              uint4* o4 = reinterpret_cast<uint4*>(static_cast<uint16_t*>(ep.out) + row * ep.ld_out + col);
              const bool f16 = ep.out_dtype == NIMBLE_DTYPE_F16;
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                float w[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) w[e] = v[8 * q + e];
                if (ep.accum_out) {
                  const uint4 a = o4[q];
                  const uint32_t av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    const uint16_t lo = av[e] & 0xFFFF, hi = av[e] >> 16;
                    w[2 * e] += f16 ? __half2float(__ushort_as_half(lo)) : __bfloat162float(__ushort_as_bfloat16(lo));
                    w[2 * e + 1] += f16 ? __half2float(__ushort_as_half(hi)) : __bfloat162float(__ushort_as_bfloat16(hi));
                  }
                }
                uint4 u;
                if (f16) {
                  u.x = pack2(__float2half_rn(w[0]), __float2half_rn(w[1]));
                  u.y = pack2(__float2half_rn(w[2]), __float2half_rn(w[3]));
                  u.z = pack2(__float2half_rn(w[4]), __float2half_rn(w[5]));
                  u.w = pack2(__float2half_rn(w[6]), __float2half_rn(w[7]));
                } else {
                  u.x = pack2(__float2bfloat16_rn(w[0]), __float2bfloat16_rn(w[1]));
                  u.y = pack2(__float2bfloat16_rn(w[2]), __float2bfloat16_rn(w[3]));
                  u.z = pack2(__float2bfloat16_rn(w[4]), __float2bfloat16_rn(w[5]));
                  u.w = pack2(__float2bfloat16_rn(w[6]), __float2bfloat16_rn(w[7]));
                }
                o4[q] = u;
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (j >= nv) break;
              float x = v[j];
              if (ep.src) x += ep.src[row * ep.ld_src + col + j];
              x *= alpha;
              const int64_t oi = row * ep.ld_out + col + j;
              if (ep.accum_out) x += load_out_elem(ep.out, oi, ep.out_dtype);
              store_out_elem(ep.out, oi, ep.out_dtype, x);
            }
          }
        }
      }
      }  // row blocks
      release(acc);
    }
    // Every G store must have landed before the CTA exits.
    if constexpr (EPI == EPI_CE_GRAD) {
      if (lane == 0) ptx::bulk_wait<0>();
      __syncwarp();
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  __syncwarp();
  // Neither CTA of a pair may leave while the other can still touch its
  // shared memory, barriers or TMEM.
  if constexpr (kCG == 2) ptx::cluster_sync();
  if (threadIdx.x == 0 && *abort_flag && ep.status) atomicOr(ep.status, NIMBLE_STATUS_WAIT_TIMEOUT);
  if (warp == 1) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc_cg<kCG>(tmem_base, kTmemCols);
  }
}

// --------------------------------------------------------- helper kernels

// Merges the per-tile (max, sum-exp) pairs of each row into the shard's row
// statistics and picks the target logit when the label lies in the shard.
__global__ void ce_row_reduce_kernel(const float2* __restrict__ part, int n_tiles, const float* __restrict__ tgt,
                                     const int64_t* __restrict__ labels, int64_t M, int64_t v_offset,
                                     int64_t v_local, float* __restrict__ out_max, float* __restrict__ out_sumexp,
                                     float* __restrict__ out_target) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= M) return;
  float m = -INFINITY, s = 0.0f;
  for (int t = 0; t < n_tiles; ++t) {
    const float2 p = part[static_cast<int64_t>(t) * M + row];
    if (p.x == -INFINITY) continue;  // a column half with no valid columns
    const float mn = fmaxf(m, p.x);
    s = s * ptx::ex2((m - mn) * kLog2e) + p.y * ptx::ex2((p.x - mn) * kLog2e);
    m = mn;
  }
  out_max[row] = m;
  out_sumexp[row] = s;
  const int64_t lab = labels[row];
  out_target[row] = (lab >= v_offset && lab < v_offset + v_local) ? tgt[row] : 0.0f;
}

// Single-block fixed-order merge of shard statistics plus the mean loss.
constexpr int kCombineThreads = 1024;
__global__ void __launch_bounds__(kCombineThreads)
ce_combine_kernel(const float* __restrict__ smax, const float* __restrict__ ssum, const float* __restrict__ stgt,
                  int P, const int64_t* __restrict__ labels, int64_t M, int64_t V, int64_t ignore_index,
                  float* __restrict__ out_max, float* __restrict__ out_sumexp, float* __restrict__ out_lse,
                  float* __restrict__ out_loss, float* __restrict__ out_valid, int* status) {
  __shared__ double s_loss[kCombineThreads];
  __shared__ int s_cnt[kCombineThreads];
  double acc = 0.0;
  int cnt = 0;
  int bad = 0;
  for (int64_t i = threadIdx.x; i < M; i += kCombineThreads) {
    float m = -INFINITY;
    for (int p = 0; p < P; ++p) m = fmaxf(m, smax[p * M + i]);
    float s = 0.0f, t = 0.0f;
    for (int p = 0; p < P; ++p) {
      s += ssum[p * M + i] * expf(smax[p * M + i] - m);
      t += stgt[p * M + i];
    }
    const float lse = m + logf(s);
    if (out_max) out_max[i] = m;
    if (out_sumexp) out_sumexp[i] = s;
    out_lse[i] = lse;
    const int64_t lab = labels[i];
    if (lab != ignore_index) {
      if (lab < 0 || lab >= V) {
        bad = 1;
      } else {
        acc += static_cast<double>(lse) - static_cast<double>(t);
        ++cnt;
      }
    }
  }
  s_loss[threadIdx.x] = acc;
  s_cnt[threadIdx.x] = cnt;
  if (bad && status) atomicOr(status, NIMBLE_STATUS_BAD_LABEL);
  // A label outside [0, V) makes the loss NaN: the caller sees it without a
  // host read of the status word (the reference raises IndexError there).
  const int any_bad = __syncthreads_or(bad);
  for (int w = kCombineThreads / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) {
      s_loss[threadIdx.x] += s_loss[threadIdx.x + w];
      s_cnt[threadIdx.x] += s_cnt[threadIdx.x + w];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const int n = s_cnt[0];
    out_loss[0] = any_bad ? __int_as_float(0x7fc00000) : (n > 0 ? static_cast<float>(s_loss[0] / n) : 0.0f);
    out_valid[0] = static_cast<float>(n);
  }
}

__global__ void round_tf32_kernel(const float* __restrict__ src, float* __restrict__ dst, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = ptx::round_tf32(src[i]);
}

// ================================================================ host side
thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}


CUtensorMapDataType tmap_dtype(int dtype) {
  if (dtype == NIMBLE_DTYPE_F32) return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  if (dtype == NIMBLE_DTYPE_F16) return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// 2-D operand map with 128-byte swizzle. K-major: a row-major [rows x k]
// matrix, boxes of box_rows x (128 bytes of K). MN-major: a row-major
// [k x mn] matrix (MN contiguous), boxes of (128 bytes of MN) x (128 / elem
// K rows). `ld` is the row pitch in elements.
int make_operand_map(CUtensorMap* map, const void* base, int dtype, bool mn_major, int64_t k, int64_t rows,
                     int64_t ld, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(NIMBLE_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled entry point unavailable");
  const int es = elem_size(dtype);
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return fail(NIMBLE_ERR_INVALID_ARG, "operand base address is not 16-byte aligned");
  if ((ld * es) % 16 != 0)
    return fail(NIMBLE_ERR_INVALID_ARG, "operand row pitch is not a multiple of 16 bytes");
  const cuuint32_t chunk = static_cast<cuuint32_t>(kBKBytes / es);
  cuuint64_t dims[2];
  cuuint32_t box[2];
  if (mn_major) {
    dims[0] = static_cast<cuuint64_t>(rows);
    dims[1] = static_cast<cuuint64_t>(k);
    box[0] = chunk;
    box[1] = chunk;
  } else {
    dims[0] = static_cast<cuuint64_t>(k);
    dims[1] = static_cast<cuuint64_t>(rows);
    box[0] = chunk;
    box[1] = static_cast<cuuint32_t>(box_rows);
  }
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * es)};
  cuuint32_t estr[2] = {1, 1};
  // MN-major fp32 (read as tf32) needs the 32-byte-atom variant of the
  // 128-byte swizzle; every other operand uses the plain 128-byte swizzle.
  const CUtensorMapSwizzle swz = (mn_major && es == 4) ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                                       : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = fn(map, tmap_dtype(dtype), 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NIMBLE_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(r));
  return NIMBLE_OK;
}

// GEMM tiling mode per GEMM kind: wide single-CTA 256 x 256 tiles by default
// (g_wide below), 128 x 256 tiles per CTA when a kind's wide bit is cleared,
// CTA pairs (cta_group::2, 256 x 256 tiles) with NIMBLEML_TIED_CE_CTA_PAIRS. The pair
// kernel keeps the tensor pipe busier per clock but draws more energy per
// FLOP, so under the B200's 1 kW cap it runs at lower clocks and is slower
// over a whole fwd+bwd step.
// The value is a bit mask over GEMM kinds: 1 forward, 2 recompute, 4 the
// store GEMMs with an MN-major A (dE), 8 the store GEMMs with a K-major A (dh);
// "1" alone keeps its historical meaning of all kinds.
const int g_cta_pairs = [] {
  const char* v = std::getenv("NIMBLEML_TIED_CE_CTA_PAIRS");
  if (!v) return 0;
  const int m = std::atoi(v);
  return m == 1 ? 15 : m;
}();
// Wide single-CTA 256 x 256 tiles, same bit mask (NIMBLEML_TIED_CE_WIDE).
// Default 15, all four GEMMs: a third fewer operand bytes per FLOP lets the
// step run at higher clocks under the power cap, which outweighs the lost
// overlap of the epilogue with the next tile's MMAs (the 8 epilogue warps
// keep that epilogue short).
const int g_wide = [] {
  const char* v = std::getenv("NIMBLEML_TIED_CE_WIDE");
  if (!v) return 15;
  const int m = std::atoi(v);
  return m == 1 ? 15 : m;
}();
constexpr int kSmemBytesWide = kStagesWide * (2 * kABytes + kBBytes) + kStoreBytes + 1024 + 256;
template <int EPI, bool kAMN>
constexpr int gemm_kind_bit() {
  return EPI == EPI_CE_FWD ? 1 : EPI == EPI_CE_GRAD ? 2 : kAMN ? 4 : 8;
}
// Token blocks per rasterisation group (NIMBLEML_TIED_CE_GROUP_M, default 8: 2048 token rows with 256-row wide tiles).
const int g_group_m = [] {
  const char* v = std::getenv("NIMBLEML_TIED_CE_GROUP_M");
  const int g = v ? std::atoi(v) : 0;
  return g > 0 ? g : 8;
}();

// Row-major [rows x cols] output written by 32 x 32 TMA box stores from a
// swizzled staging buffer (64-byte swizzle for 16-bit rows of 64 B, 128-byte
// swizzle for fp32 rows of 128 B).
int make_store_map(CUtensorMap* map, const void* base, int dtype, int64_t cols, int64_t rows, int64_t ld) {
  auto fn = encode_fn();
  if (!fn) return fail(NIMBLE_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled entry point unavailable");
  const int es = elem_size(dtype);
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld * es) % 16 != 0)
    return fail(NIMBLE_ERR_INVALID_ARG, "store target is not 16-byte aligned");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * es)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, tmap_dtype(dtype), 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, es == 2 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NIMBLE_ERR_CUDA, "cuTensorMapEncodeTiled (store) failed: " + std::to_string(r));
  return NIMBLE_OK;
}

struct DevInfo {
  int sms = 0;
  int major = 0;
};

int device_info(DevInfo* info) {
  int dev = 0;
  NIMBLE_CUDA_TRY(cudaGetDevice(&dev));
  // cuTensorMapEncodeTiled is a driver call and needs a current context; a
  // fresh host thread (e.g. torch's autograd worker) may not have one yet.
  // cudaSetDevice makes the device's primary context current on this thread.
  thread_local int ctx_dev = -1;
  if (ctx_dev != dev) {
    NIMBLE_CUDA_TRY(cudaSetDevice(dev));
    ctx_dev = dev;
  }
  NIMBLE_CUDA_TRY(cudaDeviceGetAttribute(&info->sms, cudaDevAttrMultiProcessorCount, dev));
  NIMBLE_CUDA_TRY(cudaDeviceGetAttribute(&info->major, cudaDevAttrComputeCapabilityMajor, dev));
  if (info->major != 10) return fail(NIMBLE_ERR_UNSUPPORTED, "requires a compute capability 10.x (B200) device");
  return NIMBLE_OK;
}

// C[M x N] = A[M x K] . B[N x K]^T with the given epilogue. A is stored
// row-major [M x K] (K-major) or [K x M] (kAMN); likewise B.
template <typename T, int EPI, bool kAMN, bool kBMN>
int launch_gemm(const void* A, int64_t lda, const void* B, int64_t ldb, int64_t M, int64_t N, int64_t K, int dtype,
                const EpiParams& ep, cudaStream_t stream, int max_ctas) {
  if (M <= 0 || N <= 0 || K <= 0) return NIMBLE_OK;
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return fail(NIMBLE_ERR_INVALID_ARG, "GEMM extent exceeds 2^31");
  DevInfo di;
  if (int rc = device_info(&di)) return rc;
  // A cap leaves SMs free for work that should overlap this GEMM (NCCL).
  if (max_ctas > 0 && max_ctas < di.sms) di.sms = max_ctas;
  CUtensorMap ma, mb, mc;
  if (int rc = make_operand_map(&ma, A, dtype, kAMN, K, M, lda, kBM)) return rc;
  if constexpr (EPI == EPI_CE_GRAD) {
    if (int rc = make_store_map(&mc, ep.g, dtype, N, M, ep.ldg)) return rc;
  } else {
    mc = ma;  // unused by the other epilogues
  }
  const bool pairs = (g_cta_pairs & gemm_kind_bit<EPI, kAMN>()) != 0;
  if (int rc = make_operand_map(&mb, B, dtype, kBMN, K, N, ldb, pairs ? kBN / 2 : kBN)) return rc;
  const int group_m = g_group_m;
  if (pairs) {
    // CTA pairs: 256 x 256 tiles, one cluster of 2 CTAs per SM pair.
    auto kern = tc_gemm_tn_kernel<T, EPI, kAMN, kBMN, 2>;
    NIMBLE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytesPair));
    const int64_t tiles = ((M + 2 * kBM - 1) / (2 * kBM)) * ((N + kBN - 1) / kBN);
    if (tiles > INT32_MAX) return fail(NIMBLE_ERR_INVALID_ARG, "too many tiles");
    const int pairs = static_cast<int>(std::min<int64_t>(tiles, di.sms / 2));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytesPair;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    NIMBLE_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, ma, mb, mc, static_cast<int>(M), static_cast<int>(N),
                                       static_cast<int>(K), group_m, ep));
  } else if (g_wide & gemm_kind_bit<EPI, kAMN>()) {
    auto kern = tc_gemm_tn_kernel<T, EPI, kAMN, kBMN, 1, true>;
    NIMBLE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytesWide));
    const int64_t tiles = ((M + 2 * kBM - 1) / (2 * kBM)) * ((N + kBN - 1) / kBN);
    if (tiles > INT32_MAX) return fail(NIMBLE_ERR_INVALID_ARG, "too many tiles");
    const int grid = static_cast<int>(std::min<int64_t>(tiles, di.sms));
    kern<<<grid, kThreads, kSmemBytesWide, stream>>>(ma, mb, mc, static_cast<int>(M), static_cast<int>(N),
                                                      static_cast<int>(K), group_m, ep);
  } else {
    auto kern = tc_gemm_tn_kernel<T, EPI, kAMN, kBMN, 1>;
    NIMBLE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    const int64_t tiles = ((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
    if (tiles > INT32_MAX) return fail(NIMBLE_ERR_INVALID_ARG, "too many tiles");
    const int grid = static_cast<int>(std::min<int64_t>(tiles, di.sms));
    kern<<<grid, kThreads, kSmemBytes, stream>>>(ma, mb, mc, static_cast<int>(M), static_cast<int>(N),
                                                  static_cast<int>(K), group_m, ep);
  }
  NIMBLE_CUDA_TRY(cudaGetLastError());
  return NIMBLE_OK;
}

template <int EPI, bool kAMN = false, bool kBMN = false>
int gemm_dispatch(int dtype, const void* A, int64_t lda, const void* B, int64_t ldb, int64_t M, int64_t N,
                  int64_t K, const EpiParams& ep, cudaStream_t s, int max_ctas = 0) {
  switch (dtype) {
    case NIMBLE_DTYPE_F16:
      return launch_gemm<__half, EPI, kAMN, kBMN>(A, lda, B, ldb, M, N, K, dtype, ep, s, max_ctas);
    case NIMBLE_DTYPE_BF16:
      return launch_gemm<__nv_bfloat16, EPI, kAMN, kBMN>(A, lda, B, ldb, M, N, K, dtype, ep, s, max_ctas);
    case NIMBLE_DTYPE_F32:
      return launch_gemm<float, EPI, kAMN, kBMN>(A, lda, B, ldb, M, N, K, dtype, ep, s, max_ctas);
  }
  return fail(NIMBLE_ERR_INVALID_ARG, "unknown dtype");
}

int launch_round(const float* src, float* dst, int64_t n, cudaStream_t s) {
  if (n <= 0) return NIMBLE_OK;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 16);
  round_tf32_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(src, dst, n);
  NIMBLE_CUDA_TRY(cudaGetLastError());
  return NIMBLE_OK;
}

constexpr size_t kAlign = 256;
size_t align_up(size_t x, size_t a = kAlign) { return (x + a - 1) / a * a; }
int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

// Forward workspace: per-tile pairs, target logits, and (fp32) tf32-rounded
// copies of the operands.
struct FwdLayout {
  size_t part = 0, tgt = 0, hr = 0, er = 0, total = 0;
};
FwdLayout fwd_layout(int64_t N, int64_t d, int64_t V, int dtype) {
  FwdLayout L;
  const int64_t n_parts = (V + kBN - 1) / kBN * kColHalves;  // one pair per tile and column half
  size_t off = 0;
  L.part = off; off = align_up(off + sizeof(float2) * n_parts * N);
  L.tgt = off; off = align_up(off + sizeof(float) * N);
  if (dtype == NIMBLE_DTYPE_F32) {  // NIMBLE_DTYPE_TF32 inputs are used in place
    L.hr = off; off = align_up(off + sizeof(float) * N * d);
    L.er = off; off = align_up(off + sizeof(float) * V * d);
  }
  L.total = off;
  return L;
}

constexpr size_t kDefaultSlabBytes = size_t(2) << 30;

// Backward workspace: the G slab (N x slab columns), an fp32 dh accumulator
// when the shard needs more than one slab, and (fp32) tf32-rounded operands.
struct BwdLayout {
  int64_t slab = 0, n_slabs = 0;
  size_t g = 0, dh = 0, hr = 0, er = 0, total = 0;
};
// `whole_vocab`: the shard may be the entire vocabulary (one GPU), so the
// backward walks it in at least two slabs and no G buffer ever holds more
// than half of the N x V logits. A shard of a vocabulary split over P >= 2
// ranks is at most half of it already; its slabs follow the byte budget
// alone, so a shard whose G fits the budget is one slab and needs no fp32
// grad_hidden accumulator.
BwdLayout bwd_layout(int64_t N, int64_t d, int64_t V, int dtype, size_t slab_bytes, bool whole_vocab = true) {
  BwdLayout L;
  const int64_t es = elem_size(dtype);
  if (slab_bytes == 0) slab_bytes = kDefaultSlabBytes;
  int64_t cols = static_cast<int64_t>(slab_bytes / (es * std::max<int64_t>(N, 1)));
  cols = std::max<int64_t>(kBN, cols / kBN * kBN);
  cols = std::min<int64_t>(cols, whole_vocab ? round_up((V + 1) / 2, kBN) : round_up(V, kBN));
  L.slab = cols;
  L.n_slabs = (V + cols - 1) / cols;
  size_t off = 0;
  L.g = off; off = align_up(off + es * N * cols);
  if (L.n_slabs > 1) { L.dh = off; off = align_up(off + sizeof(float) * N * d); }
  if (dtype == NIMBLE_DTYPE_F32) {  // NIMBLE_DTYPE_TF32 inputs are used in place
    L.hr = off; off = align_up(off + sizeof(float) * N * d);
    L.er = off; off = align_up(off + sizeof(float) * V * d);
  }
  L.total = off;
  return L;
}

// Shape / dtype / pointer checks shared by the entry points; `labels` may be
// null when the entry point takes none (the tied-logits GEMMs).
int check_common(const void* h, const void* w, const int64_t* labels, int64_t N, int64_t d, int64_t V, int dtype,
                 bool needs_labels = true, bool allow_tf32 = false) {
  if (dtype != NIMBLE_DTYPE_F32 && dtype != NIMBLE_DTYPE_F16 && dtype != NIMBLE_DTYPE_BF16 &&
      !(allow_tf32 && dtype == NIMBLE_DTYPE_TF32))
    return fail(NIMBLE_ERR_INVALID_ARG, allow_tf32 ? "dtype must be NIMBLE_DTYPE_F32, F16, BF16 or TF32"
                                                   : "dtype must be NIMBLE_DTYPE_F32, F16 or BF16");
  if (N < 0 || d <= 0 || V <= 0) return fail(NIMBLE_ERR_INVALID_ARG, "sizes must be positive");
  if ((d * elem_size(dtype)) % 16 != 0)
    return fail(NIMBLE_ERR_INVALID_ARG, "d_model * element size must be a multiple of 16 bytes");
  if (N > 0 && (!h || !w || (needs_labels && !labels))) return fail(NIMBLE_ERR_INVALID_ARG, "null input pointer");
  return NIMBLE_OK;
}

}  // namespace
}  // namespace nimble

// ================================================================== C ABI
using namespace nimble;

extern "C" int nimble_tied_ce_available(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return 0;
  }
  for (int i = 0; i < n; ++i) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, i) == cudaSuccess && major == 10)
      return 1;
  }
  return 0;
}

extern "C" const char* nimble_tied_ce_last_error(void) { return g_last_error.c_str(); }

extern "C" int nimble_tied_ce_forward_workspace_size(int64_t n_tokens, int64_t d_model, int64_t v_local, int dtype,
                                                     size_t* bytes) {
  if (!bytes) return fail(NIMBLE_ERR_INVALID_ARG, "bytes is null");
  if (n_tokens < 0 || d_model <= 0 || v_local <= 0) return fail(NIMBLE_ERR_INVALID_ARG, "sizes must be positive");
  *bytes = fwd_layout(n_tokens, d_model, v_local, dtype).total;
  return NIMBLE_OK;
}

extern "C" int nimble_tied_ce_forward(const void* hidden, const void* weights, const int64_t* labels, int64_t n_tokens,
                                      int64_t d_model, int64_t v_local, int64_t v_offset, int dtype, float* shard_max,
                                      float* shard_sumexp, float* shard_target, void* workspace,
                                      size_t workspace_bytes, int* status, void* stream) {
  if (int rc = check_common(hidden, weights, labels, n_tokens, d_model, v_local, dtype, true, true)) return rc;
  if (n_tokens == 0) return NIMBLE_OK;
  if (!shard_max || !shard_sumexp || !shard_target) return fail(NIMBLE_ERR_INVALID_ARG, "null output pointer");
  const FwdLayout L = fwd_layout(n_tokens, d_model, v_local, dtype);
  if (!workspace || workspace_bytes < L.total) return fail(NIMBLE_ERR_WORKSPACE, "forward workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const void* A = hidden;
  const void* B = weights;
  if (dtype == NIMBLE_DTYPE_F32) {
    float* hr = reinterpret_cast<float*>(ws + L.hr);
    float* er = reinterpret_cast<float*>(ws + L.er);
    if (int rc = launch_round(static_cast<const float*>(hidden), hr, n_tokens * d_model, s)) return rc;
    if (int rc = launch_round(static_cast<const float*>(weights), er, v_local * d_model, s)) return rc;
    A = hr;
    B = er;
  }
  if (dtype == NIMBLE_DTYPE_TF32) dtype = NIMBLE_DTYPE_F32;  // already rounded: read in place
  EpiParams ep{};
  ep.labels = labels;
  ep.col_origin = v_offset;
  ep.part = reinterpret_cast<float2*>(ws + L.part);
  ep.tgt = reinterpret_cast<float*>(ws + L.tgt);
  ep.status = status;
  if (int rc = gemm_dispatch<EPI_CE_FWD>(dtype, A, d_model, B, d_model, n_tokens, v_local, d_model, ep, s)) return rc;
  const int n_parts = static_cast<int>((v_local + kBN - 1) / kBN * kColHalves);
  ce_row_reduce_kernel<<<static_cast<unsigned>((n_tokens + 255) / 256), 256, 0, s>>>(
      ep.part, n_parts, ep.tgt, labels, n_tokens, v_offset, v_local, shard_max, shard_sumexp, shard_target);
  NIMBLE_CUDA_TRY(cudaGetLastError());
  return NIMBLE_OK;
}

extern "C" int nimble_tied_ce_combine(const float* shard_max, const float* shard_sumexp, const float* shard_target,
                                      int n_shards, const int64_t* labels, int64_t n_tokens, int64_t vocab_size,
                                      int64_t ignore_index, float* out_max, float* out_sumexp, float* out_lse,
                                      float* out_loss, float* out_valid_count, int* status, void* stream) {
  if (n_shards <= 0 || n_tokens < 0 || vocab_size <= 0) return fail(NIMBLE_ERR_INVALID_ARG, "bad sizes");
  if (!out_loss || !out_valid_count || (n_tokens > 0 && !out_lse))
    return fail(NIMBLE_ERR_INVALID_ARG, "null output pointer");
  if (n_tokens > 0 && (!shard_max || !shard_sumexp || !shard_target || !labels))
    return fail(NIMBLE_ERR_INVALID_ARG, "null input pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ce_combine_kernel<<<1, kCombineThreads, 0, s>>>(shard_max, shard_sumexp, shard_target, n_shards, labels, n_tokens,
                                                  vocab_size, ignore_index, out_max, out_sumexp, out_lse, out_loss,
                                                  out_valid_count, status);
  NIMBLE_CUDA_TRY(cudaGetLastError());
  return NIMBLE_OK;
}

extern "C" int nimble_tied_ce_backward_workspace_size(int64_t n_tokens, int64_t d_model, int64_t v_local, int dtype,
                                                      size_t slab_bytes, size_t* bytes) {
  if (!bytes) return fail(NIMBLE_ERR_INVALID_ARG, "bytes is null");
  if (n_tokens < 0 || d_model <= 0 || v_local <= 0) return fail(NIMBLE_ERR_INVALID_ARG, "sizes must be positive");
  *bytes = bwd_layout(n_tokens, d_model, v_local, dtype, slab_bytes).total;
  return NIMBLE_OK;
}

extern "C" int nimble_tied_ce_backward_overlap_workspace_size(int64_t n_tokens, int64_t d_model, int64_t v_local,
                                                              int dtype, size_t slab_bytes, size_t* bytes) {
  if (!bytes) return fail(NIMBLE_ERR_INVALID_ARG, "bytes is null");
  if (n_tokens < 0 || d_model <= 0 || v_local <= 0) return fail(NIMBLE_ERR_INVALID_ARG, "sizes must be positive");
  *bytes = bwd_layout(n_tokens, d_model, v_local, dtype, slab_bytes, /*whole_vocab=*/false).total;
  return NIMBLE_OK;
}

extern "C" int nimble_round_tf32(const float* src, float* dst, int64_t n, void* stream) {
  if (n < 0) return fail(NIMBLE_ERR_INVALID_ARG, "n must be >= 0");
  if (n > 0 && (!src || !dst)) return fail(NIMBLE_ERR_INVALID_ARG, "null pointer argument");
  return launch_round(src, dst, n, static_cast<cudaStream_t>(stream));
}

namespace {
int backward_impl(const float* grad_scale, const void* hidden, const void* weights, const int64_t* labels,
                  const float* lse, const float* valid_count, int64_t n_tokens, int64_t d_model, int64_t v_local,
                  int64_t v_offset, int64_t ignore_index, int dtype, void* grad_hidden, int grad_hidden_dtype,
                  void* grad_weights, int grad_weights_dtype, int accumulate_grad_weights, size_t slab_bytes,
                  void* workspace, size_t workspace_bytes, int* status, void* stream, void* dh_done_event,
                  int last_de_max_ctas, float capped_fraction) {
  if (int rc = check_common(hidden, weights, labels, n_tokens, d_model, v_local, dtype, true, true)) return rc;
  if (!grad_weights || !grad_scale || !valid_count || (n_tokens > 0 && (!grad_hidden || !lse)))
    return fail(NIMBLE_ERR_INVALID_ARG, "null pointer argument");
  for (int dt : {grad_hidden_dtype, grad_weights_dtype})
    if (dt != NIMBLE_DTYPE_F32 && dt != NIMBLE_DTYPE_F16 && dt != NIMBLE_DTYPE_BF16)
      return fail(NIMBLE_ERR_INVALID_ARG, "bad output dtype");
  if ((reinterpret_cast<uintptr_t>(grad_hidden) & 15) || (reinterpret_cast<uintptr_t>(grad_weights) & 15))
    return fail(NIMBLE_ERR_INVALID_ARG, "gradient outputs must be 16-byte aligned");
  if ((d_model * elem_size(grad_hidden_dtype)) % 16 || (d_model * elem_size(grad_weights_dtype)) % 16)
    return fail(NIMBLE_ERR_INVALID_ARG, "d_model * output element size must be a multiple of 16 bytes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_tokens == 0) {
    if (!accumulate_grad_weights)
      NIMBLE_CUDA_TRY(cudaMemsetAsync(grad_weights, 0, elem_size(grad_weights_dtype) * v_local * d_model, s));
    return NIMBLE_OK;
  }
  const BwdLayout L = bwd_layout(n_tokens, d_model, v_local, dtype, slab_bytes, /*whole_vocab=*/!dh_done_event);
  if (!workspace || workspace_bytes < L.total) return fail(NIMBLE_ERR_WORKSPACE, "backward workspace too small");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int64_t es = elem_size(dtype);
  const void* h = hidden;
  const void* E = weights;
  if (dtype == NIMBLE_DTYPE_F32) {
    float* hr = reinterpret_cast<float*>(ws + L.hr);
    float* er = reinterpret_cast<float*>(ws + L.er);
    if (int rc = launch_round(static_cast<const float*>(hidden), hr, n_tokens * d_model, s)) return rc;
    if (int rc = launch_round(static_cast<const float*>(weights), er, v_local * d_model, s)) return rc;
    h = hr;
    E = er;
  }
  if (dtype == NIMBLE_DTYPE_TF32) dtype = NIMBLE_DTYPE_F32;  // already rounded: read in place
  void* g = ws + L.g;
  float* dh_acc = L.n_slabs > 1 ? reinterpret_cast<float*>(ws + L.dh) : nullptr;

  // G is stored scaled by 2^15 in fp16 so that softmax probabilities of order
  // 1/V stay in the normal range; the scale is undone in the dE / dh epilogue.
  const float gscale = dtype == NIMBLE_DTYPE_F16 ? 32768.0f : 1.0f;
  for (int64_t sl = 0; sl < L.n_slabs; ++sl) {
    const int64_t c0 = sl * L.slab;
    const int64_t vc = std::min<int64_t>(L.slab, v_local - c0);
    const void* E_sl = static_cast<const uint8_t*>(E) + es * c0 * d_model;
    // 1) recompute the slab's logits, write G [N x vc] (row pitch L.slab).
    EpiParams eg{};
    eg.labels = labels;
    eg.col_origin = v_offset + c0;
    eg.ignore_index = ignore_index;
    eg.lse = lse;
    eg.g = g;
    eg.ldg = L.slab;
    eg.gscale = gscale;
    eg.status = status;
    if (int rc = gemm_dispatch<EPI_CE_GRAD>(dtype, h, d_model, E_sl, d_model, n_tokens, vc, d_model, eg, s)) return rc;
    const bool last = sl == L.n_slabs - 1;
    // 2) dE[c0:c0+vc] = G^T h: A = G read MN-major ([tokens x vc]), B = h
    //    read MN-major ([tokens x d]); K = tokens.
    // dE rows [r0, r1) of the slab on at most max_ctas SMs (0 = all).
    auto run_de = [&](int max_ctas, int64_t r0, int64_t r1) -> int {
      if (r1 <= r0) return NIMBLE_OK;
      EpiParams ee{};
      ee.out = static_cast<uint8_t*>(grad_weights) + elem_size(grad_weights_dtype) * (c0 + r0) * d_model;
      ee.ld_out = d_model;
      ee.out_dtype = grad_weights_dtype;
      ee.alpha_num = grad_scale;
      ee.alpha_den = valid_count;
      ee.alpha_mult = 1.0f / gscale;
      ee.accum_out = accumulate_grad_weights ? 1 : 0;
      ee.status = status;
      return gemm_dispatch<EPI_STORE, true, true>(dtype, static_cast<uint8_t*>(g) + es * r0, L.slab, h, d_model,
                                                  r1 - r0, d_model, n_tokens, ee, s, max_ctas);
    };
    // 3) dh (+)= G E[c0:c0+vc]: A = G K-major, B = E slab read MN-major
    //    ([vc x d]); K = slab columns.
    auto run_dh = [&]() -> int {
      EpiParams eh{};
      eh.status = status;
      if (last) {
        eh.out = grad_hidden;
        eh.out_dtype = grad_hidden_dtype;
        eh.alpha_num = grad_scale;
        eh.alpha_den = valid_count;
        eh.alpha_mult = 1.0f / gscale;
      } else {
        eh.out = dh_acc;
        eh.out_dtype = NIMBLE_DTYPE_F32;
        eh.alpha_mult = 1.0f;
      }
      eh.ld_out = d_model;
      eh.src = sl > 0 ? dh_acc : nullptr;
      eh.ld_src = d_model;
      return gemm_dispatch<EPI_STORE, false, true>(dtype, g, L.slab, E_sl, d_model, n_tokens, d_model, vc, eh, s);
    };
    if (last && dh_done_event) {
      // grad_hidden is final after this slab's dh GEMM: announce it, then
      // run the last dE GEMM (optionally on fewer SMs) while the caller
      // reduces grad_hidden across ranks.
      // Its first rows run beside the caller's reduction on fewer SMs, the
      // rest on all SMs once the reduction is expected to be done.
      if (int rc = run_dh()) return rc;
      NIMBLE_CUDA_TRY(cudaEventRecord(static_cast<cudaEvent_t>(dh_done_event), s));
      int64_t split = vc;
      if (capped_fraction < 1.0f)
        split = std::min<int64_t>(vc, round_up(static_cast<int64_t>(capped_fraction * static_cast<double>(vc)), kBN));
      if (int rc = run_de(last_de_max_ctas, 0, split)) return rc;
      if (int rc = run_de(0, split, vc)) return rc;
    } else {
      if (int rc = run_de(0, 0, vc)) return rc;
      if (int rc = run_dh()) return rc;
    }
  }
  return NIMBLE_OK;
}
}  // namespace

extern "C" int nimble_tied_ce_backward(const float* grad_scale, const void* hidden, const void* weights,
                                       const int64_t* labels, const float* lse, const float* valid_count,
                                       int64_t n_tokens, int64_t d_model, int64_t v_local, int64_t v_offset,
                                       int64_t ignore_index, int dtype, void* grad_hidden, int grad_hidden_dtype,
                                       void* grad_weights, int grad_weights_dtype, int accumulate_grad_weights,
                                       size_t slab_bytes, void* workspace, size_t workspace_bytes, int* status,
                                       void* stream) {
  return backward_impl(grad_scale, hidden, weights, labels, lse, valid_count, n_tokens, d_model, v_local, v_offset,
                       ignore_index, dtype, grad_hidden, grad_hidden_dtype, grad_weights, grad_weights_dtype,
                       accumulate_grad_weights, slab_bytes, workspace, workspace_bytes, status, stream, nullptr, 0,
                       1.0f);
}

extern "C" int nimble_tied_ce_backward_overlap(const float* grad_scale, const void* hidden, const void* weights,
                                               const int64_t* labels, const float* lse, const float* valid_count,
                                               int64_t n_tokens, int64_t d_model, int64_t v_local, int64_t v_offset,
                                               int64_t ignore_index, int dtype, void* grad_hidden,
                                               int grad_hidden_dtype, void* grad_weights, int grad_weights_dtype,
                                               int accumulate_grad_weights, size_t slab_bytes, void* workspace,
                                               size_t workspace_bytes, int* status, void* stream,
                                               void* grad_hidden_ready_event, int last_de_max_ctas,
                                               float capped_fraction) {
  if (!grad_hidden_ready_event) return fail(NIMBLE_ERR_INVALID_ARG, "null grad_hidden_ready_event");
  if (last_de_max_ctas < 0) return fail(NIMBLE_ERR_INVALID_ARG, "last_de_max_ctas must be >= 0");
  if (!(capped_fraction >= 0.0f)) return fail(NIMBLE_ERR_INVALID_ARG, "capped_fraction must be >= 0");
  return backward_impl(grad_scale, hidden, weights, labels, lse, valid_count, n_tokens, d_model, v_local, v_offset,
                       ignore_index, dtype, grad_hidden, grad_hidden_dtype, grad_weights, grad_weights_dtype,
                       accumulate_grad_weights, slab_bytes, workspace, workspace_bytes, status, stream,
                       grad_hidden_ready_event, last_de_max_ctas, capped_fraction);
}

// ================================================================ diagnostics
// One block waits on an mbarrier that nothing will ever arrive on, through the
// same bounded wait the GEMM pipeline uses; it must give up after limit_ns,
// report NIMBLE_STATUS_WAIT_TIMEOUT and leave the context usable.
__global__ void wait_timeout_probe_kernel(int* status, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    ptx::mbar_init(&bar, 1);
    abort_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();
  const bool ok = ptx::mbar_wait(&bar, 0, &abort_flag, limit_ns);
  __syncthreads();
  if (threadIdx.x == 0 && (!ok || abort_flag)) atomicOr(status, NIMBLE_STATUS_WAIT_TIMEOUT);
}

extern "C" int nimble_tied_ce_probe_wait_timeout(uint64_t limit_ns, int* status, void* stream) {
  if (!status) return fail(NIMBLE_ERR_INVALID_ARG, "null status");
  if (limit_ns == 0 || limit_ns > ptx::kWaitLimitNs) return fail(NIMBLE_ERR_INVALID_ARG, "limit_ns must be in (0, 2 s]");
  wait_timeout_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, limit_ns);
  NIMBLE_CUDA_TRY(cudaGetLastError());
  return NIMBLE_OK;
}

// ======================================================== tied LM-head logits
// Materialised logits of the tied head for evaluation and generation
// (the reference's GPT.forward / _tied_logits), on the same tcgen05 GEMM with
// the plain store epilogue.

extern "C" int nimble_tied_logits_forward(const void* hidden, int64_t hidden_row_pitch, const void* weights,
                                          int64_t n_rows, int64_t d_model, int64_t vocab, int dtype,
                                          void* logits, int64_t logits_row_pitch, int logits_dtype,
                                          void* stream) {
  if (int rc = check_common(hidden, weights, nullptr, n_rows, d_model, vocab, dtype, /*needs_labels=*/false))
    return rc;
  if (n_rows == 0) return NIMBLE_OK;
  if (!logits) return fail(NIMBLE_ERR_INVALID_ARG, "null logits pointer");
  if (logits_dtype != NIMBLE_DTYPE_F32 && logits_dtype != NIMBLE_DTYPE_F16 && logits_dtype != NIMBLE_DTYPE_BF16)
    return fail(NIMBLE_ERR_INVALID_ARG, "bad logits dtype");
  if (hidden_row_pitch < d_model) return fail(NIMBLE_ERR_INVALID_ARG, "hidden_row_pitch must be >= d_model");
  if (logits_row_pitch < vocab) return fail(NIMBLE_ERR_INVALID_ARG, "logits_row_pitch must be >= vocab");
  if ((reinterpret_cast<uintptr_t>(logits) & 15) || (logits_row_pitch * elem_size(logits_dtype)) % 16)
    return fail(NIMBLE_ERR_INVALID_ARG, "logits must be 16-byte aligned with a row pitch of a multiple of 16 bytes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == NIMBLE_DTYPE_F32)
    return fail(NIMBLE_ERR_INVALID_ARG, "tied logits support f16 / bf16 compute");
  EpiParams ep{};
  ep.out = logits;
  ep.ld_out = logits_row_pitch;
  ep.out_dtype = logits_dtype;
  ep.alpha_mult = 1.0f;
  return gemm_dispatch<EPI_STORE>(dtype, hidden, hidden_row_pitch, weights, d_model, n_rows, vocab, d_model, ep, s);
}

extern "C" int nimble_tied_logits_backward(const void* grad_logits, int64_t grad_logits_row_pitch,
                                           const void* hidden, const void* weights,
                                           int64_t n_rows, int64_t d_model, int64_t vocab, int dtype,
                                           void* grad_hidden, int grad_hidden_dtype, void* grad_weights,
                                           int grad_weights_dtype, int accumulate_grad_weights, void* stream) {
  if (int rc = check_common(hidden, weights, nullptr, n_rows, d_model, vocab, dtype, /*needs_labels=*/false))
    return rc;
  if (dtype == NIMBLE_DTYPE_F32)
    return fail(NIMBLE_ERR_INVALID_ARG, "tied logits support f16 / bf16 compute");
  if (n_rows > 0 && !grad_logits) return fail(NIMBLE_ERR_INVALID_ARG, "null grad_logits");
  if (grad_logits_row_pitch < vocab) return fail(NIMBLE_ERR_INVALID_ARG, "grad_logits_row_pitch must be >= vocab");
  for (int dt : {grad_hidden_dtype, grad_weights_dtype})
    if (dt != NIMBLE_DTYPE_F32 && dt != NIMBLE_DTYPE_F16 && dt != NIMBLE_DTYPE_BF16)
      return fail(NIMBLE_ERR_INVALID_ARG, "bad output dtype");
  if ((grad_hidden && (reinterpret_cast<uintptr_t>(grad_hidden) & 15)) ||
      (grad_weights && (reinterpret_cast<uintptr_t>(grad_weights) & 15)))
    return fail(NIMBLE_ERR_INVALID_ARG, "gradient outputs must be 16-byte aligned");
  if ((d_model * elem_size(grad_hidden_dtype)) % 16 || (d_model * elem_size(grad_weights_dtype)) % 16)
    return fail(NIMBLE_ERR_INVALID_ARG, "d_model * output element size must be a multiple of 16 bytes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (grad_weights && n_rows == 0) {
    if (!accumulate_grad_weights)
      NIMBLE_CUDA_TRY(cudaMemsetAsync(grad_weights, 0, elem_size(grad_weights_dtype) * vocab * d_model, s));
    return NIMBLE_OK;
  }
  if (grad_hidden) {
    // grad_hidden = grad_logits . E: A = grad_logits K-major, B = E MN-major.
    EpiParams eh{};
    eh.out = grad_hidden;
    eh.ld_out = d_model;
    eh.out_dtype = grad_hidden_dtype;
    eh.alpha_mult = 1.0f;
    if (int rc = gemm_dispatch<EPI_STORE, false, true>(dtype, grad_logits, grad_logits_row_pitch, weights, d_model, n_rows, d_model,
                                                       vocab, eh, s))
      return rc;
  }
  if (grad_weights) {
    // grad_weights (+)= grad_logits^T . hidden: both operands MN-major.
    EpiParams ew{};
    ew.out = grad_weights;
    ew.ld_out = d_model;
    ew.out_dtype = grad_weights_dtype;
    ew.alpha_mult = 1.0f;
    ew.accum_out = accumulate_grad_weights ? 1 : 0;
    if (int rc = gemm_dispatch<EPI_STORE, true, true>(dtype, grad_logits, grad_logits_row_pitch, hidden, d_model, vocab, d_model,
                                                      n_rows, ew, s))
      return rc;
  }
  return NIMBLE_OK;
}

// ============================================ allocation-free forward variant
// For callers that cannot allocate device memory at all: e.g. a host runtime
// whose GPU memory is owned by another framework's pool, or an embedding
// layer that may only hand over tensors it already holds. The forward's
// per-tile scratch then lives in this fixed file-scope array instead of a
// caller workspace. Every GPU that loads this library keeps the array
// resident until the process exits.
namespace nimble {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;  // 64 MiB
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the scratch array on the current device. In host code
// the symbol is only a host-side stand-in, so the address is looked up with
// the device current. It is looked up on every call (no allocation, no
// cached pointer), so it stays right after cudaDeviceReset or a reload of
// the module.
int noalloc_scratch(void** out) {
  void* p = nullptr;
  NIMBLE_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
  *out = p;
  return NIMBLE_OK;
}

}  // namespace
}  // namespace nimble

extern "C" int nimble_tied_ce_forward_noalloc(const void* hidden, const void* weights, const int64_t* labels,
                                              int64_t n_tokens, int64_t d_model, int64_t v_local,
                                              int64_t v_offset, int dtype, float* shard_max, float* shard_sumexp,
                                              float* shard_target, int* status, void* stream) {
  if (int rc = check_common(hidden, weights, labels, n_tokens, d_model, v_local, dtype, true, true)) return rc;
  const size_t need = fwd_layout(n_tokens, d_model, v_local, dtype).total;
  if (need > kNoAllocScratchBytes)
    return fail(NIMBLE_ERR_INVALID_ARG,
                "nimble_tied_ce_forward_noalloc: these sizes need " + std::to_string(need) +
                    " bytes of scratch but the built-in array holds " + std::to_string(kNoAllocScratchBytes) +
                    " (64 MiB); split the tokens into smaller calls or use nimble_tied_ce_forward");
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  // Nothing in the scratch needs to start at zero: every per-tile pair is
  // written before the row reduce reads it, and a row's target slot is only
  // read when the tile that owns its label wrote it in this call.
  return nimble_tied_ce_forward(hidden, weights, labels, n_tokens, d_model, v_local, v_offset, dtype, shard_max,
                                shard_sumexp, shard_target, scratch, kNoAllocScratchBytes, status, stream);
}
