// Two-SM variant of the tcgen05 GEMM: a cluster of two CTAs computes one
// 256 x 256 tile with tcgen05.mma.cta_group::2 (M = 256 across the pair).
//
// * Each CTA loads, by TMA into its own shared memory, its 128 rows of A and
//   its half (128 rows) of B; both loads signal the leader CTA's full barrier
//   (the leader arms it with both CTAs' bytes). No multicast: every CTA
//   fetches its own tiles.
// * The leader's elected thread issues the pair MMAs; their commits arrive on
//   the stage-empty and accumulator-full barriers of both CTAs.
// * Each CTA's eight epilogue warps drain its own TMEM (its 128 rows of the
//   tile, all 256 columns) with the same fused epilogue as the one-SM kernel,
//   then release the accumulator on the leader's barrier.
// Per SM and 64-element k-block this moves 32 KB of operands for 4 MFLOP
// (half of the one-SM 128x256 tile's 48 KB), the reason for the pair. A
// pipeline stage holds two such k-blocks (two 128-byte swizzle atoms of K,
// 64 KB per CTA, three stages): half as many barrier round trips per FLOP as
// one atom per stage, measured 3 % faster on the Newton-Schulz step.
#pragma once

#include "gemm.cuh"

namespace po {

template <int KIND, int ATOMS_ = 2>
struct PairCfg {
  static constexpr int TM = 256;                          // rows per pair tile
  static constexpr int BN = 256;                          // columns per tile
  static constexpr int ES = (KIND == KIND_BF16) ? 2 : 4;
  static constexpr int ATOMS = ATOMS_;                    // 128-byte swizzle atoms of K per stage
  static constexpr int AK = 128 / ES;                     // K elements per atom
  static constexpr int BK = ATOMS * AK;
  static constexpr int A_BYTES = 128 * 128 * ATOMS;       // this CTA's 128 rows of A
  static constexpr int B_BYTES = (BN / 2) * 128 * ATOMS;  // this CTA's half of B
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;   // per CTA
  static constexpr int STAGES = 6 / ATOMS;               // 192 KB of stages per CTA either way
  static constexpr int MMA_K = (KIND == KIND_BF16) ? 16 : 8;
  static constexpr int KSTEPS = BK / MMA_K;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 512;
  static_assert(SMEM_BYTES <= 232448, "shared memory");
};

constexpr int kPairEpilogueWarps = 16;  // eight per CTA, each releases once per tile

// Tile queue. The leader's producer thread takes tile indices from a global
// counter (P.sched) in the order the pairs become free, so the tiles in flight
// always form one contiguous window of the raster and share their operand
// panels through L2 (a fixed round-robin lets pairs drift apart). Each index
// is published through a ring of kSchedSlots entries in both CTAs' shared
// memory; a slot is reused once all its readers have released it.
constexpr int kSchedSlots = 4;
// Readers of each slot: leader MMA issuer + 8 leader epilogue warps, peer
// producer + 8 peer epilogue warps.
constexpr int kSchedReaders = 2 + kPairEpilogueWarps;

// Reader side of the tile queue: index of the j-th tile this pair works on.
__device__ __forceinline__ bool sched_read(uint64_t* sfull, const int* stile, int j, volatile int* abort_flag,
                                           int* err, int code, int& t) {
  const int slot = j % kSchedSlots;
  if (!mbar_wait_bounded_cluster(sfull + slot, (j / kSchedSlots) & 1u, abort_flag, err, code)) return false;
  t = *reinterpret_cast<const volatile int*>(stile + slot);
  return true;
}
__device__ __forceinline__ void sched_release(uint64_t* sempty, int j) {
  mbar_arrive_cluster(mapa_shared(smem_u32(sempty + j % kSchedSlots), 0));
}

template <int KIND, bool A_MN, bool B_MN, int ATOMS>
__global__ void __launch_bounds__(kGemmThreads, 1) tc_gemm_pair_kernel(const __grid_constant__ GemmParams P) {
  using C = PairCfg<KIND, ATOMS>;
  constexpr int BN = C::BN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* sfull = drain + 1;               // [kSchedSlots] tile index published
  uint64_t* sempty = sfull + kSchedSlots;    // [kSchedSlots] all readers done (leader's copy is used)
  int* stile = reinterpret_cast<int*>(sempty + kSchedSlots);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(stile + kSchedSlots);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(cluster_id_x());
  const int npairs = static_cast<int>(cluster_count_x());

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull + a, 1);
      mbar_init(tempty + a, kPairEpilogueWarps);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < kSchedSlots; ++i) {
      mbar_init(sfull + i, 1);
      mbar_init(sempty + i, kSchedReaders);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&P.mapA[0]);
    prefetch_tensormap(&P.mapB[0]);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before_sync();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_holder;
  const int nkb = (P.K + C::BK - 1) / C::BK;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer (both CTAs)
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t armed = 0;
      const long long prof_t0 = P.prof != nullptr ? clock64() : 0;
      long long prof_empty = 0;
      for (int j = 0; ok; ++j) {
        int t;
        if (leader) {
          // Take the next tile and publish it to both CTAs.
          const int slot = j % kSchedSlots;
          if (!mbar_wait_bounded_cluster(sempty + slot, ((j / kSchedSlots) & 1u) ^ 1u, abort_flag, P.err,
                                         kErrTimeoutProducer))
            break;
          t = P.sched != nullptr ? static_cast<int>(atomicAdd(P.sched, 1u)) : pair + j * npairs;
          stile[slot] = t;
          st_shared_cluster_u32(mapa_shared(smem_u32(stile + slot), 1), static_cast<uint32_t>(t));
          mbar_arrive(sfull + slot);
          mbar_arrive_cluster(mapa_shared(smem_u32(sfull + slot), 1));
        } else {
          if (!sched_read(sfull, stile, j, abort_flag, P.err, kErrTimeoutProducer, t)) break;
          sched_release(sempty, j);
        }
        if (t >= P.total_tiles) break;
        const TileCoord tc = decode_tile(P, t);
        if (!tile_active(P, tc.b)) continue;
        const int nv = tile_passes(P, tc.b) * nkb;
        const int arow = tc.mt * C::TM + static_cast<int>(rank) * 128;
        const int brow = tc.nt * BN + static_cast<int>(rank) * (BN / 2);
        for (int v = 0; v < nv; ++v) {
          const int pass = v / nkb;
          const int k0 = (v - pass * nkb) * C::BK;
          const long long pw0 = P.prof != nullptr ? clock64() : 0;
          const bool got_empty = mbar_wait_bounded(empty + stage, phase ^ 1u, abort_flag, P.err, kErrTimeoutProducer);
          if (P.prof != nullptr) prof_empty += clock64() - pw0;
          if (!got_empty) {
            ok = false;
            break;
          }
          if (leader) {
            mbar_arrive_expect_tx(full + stage, 2 * C::STAGE_BYTES);
            armed = (armed & ~(0x101u << stage)) | (1u << stage) | (phase << (8 + stage));
          }
          const uint32_t bar = mapa_shared(smem_u32(full + stage), 0);
          const CUtensorMap* ma = &P.mapA[pass == 2 ? 1 : 0];
          const CUtensorMap* mb = &P.mapB[pass == 1 ? 1 : 0];
          uint8_t* sa = tiles + stage * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
          if (!A_MN) {
#pragma unroll
            for (int a = 0; a < C::ATOMS; ++a) tma_load_3d_pair(sa + a * 128 * 128, ma, bar, k0 + a * C::AK, arow, tc.b);
          } else if (P.a4d) {
            tma_load_4d_pair(sa, ma, bar, 0, k0, arow / (128 / C::ES), tc.b);
          } else {
#pragma unroll
            for (int i = 0; i < 128 * C::ES / 128; ++i)
              tma_load_3d_pair(sa + i * C::BK * 128, ma, bar, arow + i * (128 / C::ES), k0, tc.b);
          }
          if (!B_MN) {
#pragma unroll
            for (int a = 0; a < C::ATOMS; ++a)
              tma_load_3d_pair(sb + a * (BN / 2) * 128, mb, bar, k0 + a * C::AK, brow, tc.b);
          } else if (P.b4d) {
            tma_load_4d_pair(sb, mb, bar, 0, k0, brow / (128 / C::ES), tc.b);
          } else {
#pragma unroll
            for (int i = 0; i < (BN / 2) * C::ES / 128; ++i)
              tma_load_3d_pair(sb + i * C::BK * 128, mb, bar, brow + i * (128 / C::ES), k0, tc.b);
          }
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (P.prof != nullptr) {
        atomicAdd(P.prof + kProfProdEmptyWait, static_cast<unsigned long long>(prof_empty));
        atomicAdd(P.prof + kProfProdTotal, static_cast<unsigned long long>(clock64() - prof_t0));
      }
      if (!ok && leader) {
        // The leader's full barrier counts both CTAs' bytes: once the last
        // arming of each stage completes, no load of either CTA is in flight.
        for (int s = 0; s < C::STAGES; ++s) {
          if (!(armed & (1u << s))) continue;
          const uint32_t par = (armed >> (8 + s)) & 1u;
          const unsigned long long t0 = global_timer_ns();
          while (!mbar_try_wait(full + s, par)) {
            if (global_timer_ns() - t0 > kWaitTimeoutNs) {
              atomicCAS(P.err, 0, kErrTimeoutDrain);
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------ MMA issuer (leader CTA)
      constexpr uint32_t fmt = (KIND == KIND_BF16) ? 1u : 2u;
      constexpr uint32_t idesc = make_idesc(fmt, C::TM, BN, A_MN ? 1u : 0u, B_MN ? 1u : 0u);
      constexpr uint32_t A_STEP = A_MN ? C::MMA_K * 128 : 32;
      constexpr uint32_t B_STEP = B_MN ? C::MMA_K * 128 : 32;
      constexpr uint32_t A_LBO = A_MN ? C::BK * 128 : 16;
      constexpr uint32_t B_LBO = B_MN ? C::BK * 128 : 16;
      constexpr bool MN32 = (KIND == KIND_TF32);
      constexpr uint32_t A_LAY = (A_MN && MN32) ? kSwizzle128BAtom32B : kSwizzle128B;
      constexpr uint32_t B_LAY = (B_MN && MN32) ? kSwizzle128BAtom32B : kSwizzle128B;
      constexpr uint32_t A_SBO = (A_MN && MN32) ? 512 : 1024;
      constexpr uint32_t B_SBO = (B_MN && MN32) ? 512 : 1024;
      int stage = 0;
      uint32_t phase = 0;
      int ucount = 0;
      bool ok = true;
      const long long prof_t0 = P.prof != nullptr ? clock64() : 0;
      long long prof_full = 0, prof_tempty = 0;
      for (int j = 0; ok; ++j) {
        int t;
        if (!sched_read(sfull, stile, j, abort_flag, P.err, kErrTimeoutMma, t)) break;
        sched_release(sempty, j);
        if (t >= P.total_tiles) break;
        const TileCoord tc = decode_tile(P, t);
        if (!tile_active(P, tc.b)) continue;
        const int nv = tile_passes(P, tc.b) * nkb;
        const int acc = ucount & 1;
        const uint32_t acc_phase = (ucount >> 1) & 1;
        const long long tw0 = P.prof != nullptr ? clock64() : 0;
        const bool got_acc = mbar_wait_bounded_cluster(tempty + acc, acc_phase ^ 1u, abort_flag, P.err, kErrTimeoutMma);
        if (P.prof != nullptr) prof_tempty += clock64() - tw0;
        if (!got_acc) break;
        tc_fence_after_sync();
        const uint32_t dtmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int v = 0; v < nv; ++v) {
          const long long fw0 = P.prof != nullptr ? clock64() : 0;
          const bool got_full = mbar_wait_bounded(full + stage, phase, abort_flag, P.err, kErrTimeoutMma);
          if (P.prof != nullptr) prof_full += clock64() - fw0;
          if (!got_full) {
            ok = false;
            break;
          }
          // TMA writes and tensor-core reads are both async-proxy operations ordered
          // by the mbarrier: no tcgen05 fence is needed between them.
          const uint32_t sa = smem_u32(tiles + stage * C::STAGE_BYTES);
          const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
          for (int ks = 0; ks < C::KSTEPS; ++ks) {
            constexpr int PER = C::KSTEPS / C::ATOMS;
            const uint32_t aoff = A_MN ? ks * A_STEP : (ks / PER) * (128 * 128) + (ks % PER) * 32;
            const uint32_t boff = B_MN ? ks * B_STEP : (ks / PER) * ((BN / 2) * 128) + (ks % PER) * 32;
            const uint64_t ad = make_sw128_desc(sa + aoff, A_LBO, A_SBO, A_LAY);
            const uint64_t bd = make_sw128_desc(sb + boff, B_LBO, B_SBO, B_LAY);
            const uint32_t accumulate = (v > 0 || ks > 0) ? 1u : 0u;
            if (KIND == KIND_BF16) mma_f16_pair(dtmem, ad, bd, idesc, accumulate);
            else mma_tf32_pair(dtmem, ad, bd, idesc, accumulate);
          }
          mma_commit_pair_mc(empty + stage, 0x3);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit_pair_mc(tfull + acc, 0x3);
        ++ucount;
      }
      if (P.prof != nullptr) {
        atomicAdd(P.prof + kProfMmaFullWait, static_cast<unsigned long long>(prof_full));
        atomicAdd(P.prof + kProfMmaTemptyWait, static_cast<unsigned long long>(prof_tempty));
        atomicAdd(P.prof + kProfMmaTotal, static_cast<unsigned long long>(clock64() - prof_t0));
        atomicAdd(P.prof + kProfTiles, static_cast<unsigned long long>(ucount));
      }
      mma_commit_pair(drain);
      {
        const unsigned long long t0 = global_timer_ns();
        while (!mbar_try_wait(drain, 0)) {
          if (global_timer_ns() - t0 > kWaitTimeoutNs) {
            atomicCAS(P.err, 0, kErrTimeoutDrain);
            break;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    constexpr int HC = BN / EC / 2;
    const int c_lo = ((warp - 2) >> 2) * HC;
    int ucount = 0;
    const bool prof_on = P.prof != nullptr && warp == 2 && lane == 0;
    const long long prof_t0 = prof_on ? clock64() : 0;
    long long prof_wait = 0, prof_work = 0;
    for (int j = 0;; ++j) {
      int t;
      const bool got = sched_read(sfull, stile, j, abort_flag, P.err, kErrTimeoutEpilogue, t);
      if (!__all_sync(0xffffffffu, got)) break;
      __syncwarp();
      if (lane == 0) sched_release(sempty, j);
      if (t >= P.total_tiles) break;
      const TileCoord tc = decode_tile(P, t);
      if (!tile_active(P, tc.b)) continue;
      const int row = tc.mt * C::TM + static_cast<int>(rank) * 128 + q * 32 + lane;
      const bool mirror = P.tri && tc.mt != tc.nt;
      float red = 0.0f;
      epilogue_prefetch(P, tc.b, row, tc.nt * BN + c_lo * EC, HC * EC);
      const int acc = ucount & 1;
      const uint32_t acc_phase = (ucount >> 1) & 1;
      const long long ew0 = prof_on ? clock64() : 0;
      const bool ready = mbar_wait_bounded_sleep(tfull + acc, acc_phase, abort_flag, P.err, kErrTimeoutEpilogue);
      const long long ew1 = prof_on ? clock64() : 0;
      if (prof_on) prof_wait += ew1 - ew0;
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after_sync();
#pragma unroll 1
      for (int c = c_lo; c < c_lo + HC; ++c) {
        uint32_t r[EC];
        tmem_ld_32x16(tmem_base + lane_base + static_cast<uint32_t>(acc * BN + c * EC), r);
        tmem_ld_wait();
        float f[EC];
#pragma unroll
        for (int j = 0; j < EC; ++j) f[j] = __uint_as_float(r[j]);
        epilogue_chunk(P, tc, row, tc.nt * BN + c * EC, mirror, f, red);
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(tempty + acc), 0));
      if (prof_on) prof_work += clock64() - ew1;
      ++ucount;
      if (P.epi.red_absmax != nullptr) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) red = fmaxf(red, __shfl_xor_sync(0xffffffffu, red, o));
        if (lane == 0 && red > 0.0f)
          atomicMax(reinterpret_cast<int*>(P.epi.red_absmax) + tc.b, __float_as_int(red));
      } else if (P.epi.red_sumsq != nullptr) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) red += __shfl_xor_sync(0xffffffffu, red, o);
        if (lane == 0) atomicAdd(P.epi.red_sumsq + (P.epi.red_sumsq_shared ? 0 : tc.b), static_cast<double>(red));
      }
    }
    if (prof_on) {
      atomicAdd(P.prof + kProfEpiFullWait, static_cast<unsigned long long>(prof_wait));
      atomicAdd(P.prof + kProfEpiWork, static_cast<unsigned long long>(prof_work));
      atomicAdd(P.prof + kProfEpiTotal, static_cast<unsigned long long>(clock64() - prof_t0));
    }
  }

  __syncwarp();
  tc_fence_before_sync();
  cluster_sync();  // every MMA drained and every TMEM read done in both CTAs
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && P.sched != nullptr) {
    // The last CTA to finish re-arms the queue for the next launch that uses it.
    __threadfence();
    if (atomicAdd(P.sched + 1, 1u) == gridDim.x - 1) {
      atomicExch(P.sched, 0u);
      atomicExch(P.sched + 1, 0u);
    }
  }
}

}  // namespace po
