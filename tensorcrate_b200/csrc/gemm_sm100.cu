// gemm_sm100.cu — f16/bf16 products on the 5th-generation tensor cores:
// Kernels::matmul / matmul_add / matmul_transposed_add (kernels.rs:956-985)
// for the compact types, f32 accumulation, each output rounded once
// (compact::matmul, src/compact.rs:232-253).
//
// One persistent CTA per SM, warp-specialised:
//   warp 0      TMA producer: 128-byte-swizzled tiles of A and B into a ring
//               of shared-memory stages (cp.async.bulk.tensor; each CTA loads
//               its own tiles).
//   warp 1      allocates TMEM; one thread issues tcgen05.mma (M=128, N=BN,
//               K=16) into an f32 accumulator in TMEM and commits each stage
//               back to the producer and each finished tile to the epilogue.
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (each warp its 32
//               TMEM lanes), + C when accumulating, round, store.
// Two accumulators in TMEM let the epilogue of one tile overlap the main
// loop of the next.
//
// Operands are read where they lie: a row-major [M,K] A or [N,K] B is
// "K-major"; A stored [K,M] (Transposed::Left) or B stored [K,N] (the plain
// product) is "MN-major", which the UMMA descriptors express with their
// leading/stride byte offsets, so no transpose copy is made.
//
// Every wait on an mbarrier is bounded: on expiry the kernel records the
// failure in a device flag (read by tc_device_status), every role stops,
// in-flight copies and MMAs are waited for (again bounded) and TMEM is freed.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "gemm.cuh"

namespace tc {

__device__ int g_gemm_fault = 0;

namespace {
thread_local int t_reserved_sms = 0;
std::atomic<unsigned long long> g_wait_ns{2000000000ull};
}
void gemm_reserve_sms(int n) { t_reserved_sms = n < 0 ? 0 : n; }
int reserved_sms() { return t_reserved_sms; }

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 f16/bf16 = 128 bytes: one swizzle row
constexpr int EPI_WARPS = 4;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr uint64_t WAIT_NS = 2000000000ull;  // 2 s per wait (drains always wait this long)
constexpr uint32_t WAIT_SPINS = 1u << 30;   // and never more spins than this

// ---- PTX wrappers ----------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait for the phase of `bar` with `parity`.  False if the CTA is aborting,
// or if `limit_ns` pass first: that records the fault and starts the abort.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = now_ns();
  for (uint32_t i = 1; i < WAIT_SPINS; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 1) {  // after the first retry, then every 64
      if (*abort_flag) return false;
      if (now_ns() - t0 > limit_ns) break;
    }
  }
  *abort_flag = 1;
  atomicExch(&g_gemm_fault, 1);
  return false;
}
// The same wait with no abort check, for draining in-flight work.
__device__ __forceinline__ void mbar_drain(uint64_t *bar, uint32_t parity) {
  const uint64_t t0 = now_ns();
  for (uint32_t i = 0; i < WAIT_SPINS; ++i) {
    if (mbar_try_wait(bar, parity)) return;
    if ((i & 63u) == 0 && now_ns() - t0 > WAIT_NS) return;
  }
}
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_prefetch(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// The shared-memory matrix descriptor: start, leading and stride byte
// offsets (>> 4), version 1, 128-byte swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

constexpr int MAX_PEERS = 7;

struct Params {
  // How long a pipeline wait lasts before the CTA gives up (drains of
  // in-flight work always allow WAIT_NS).
  unsigned long long wait_ns;
  int M, N, K;
  int a_mn, b_mn;  // 1 = MN-major operand
  int accumulate;
  void *c;
  int elem_is_bf16;
  int vec_store;  // rows of C start 16-byte aligned
  // The same C on other GPUs (peer pointers over NVLink): every tile is
  // stored there as well as to `c`, which fuses an all-gather of row panels
  // into the epilogue.
  int n_peers;
  void *peer_c[MAX_PEERS];
  // Epilogue of a dense layer, in this order on the rounded product P:
  // P = round(P * MaxShare(share_of[row, col], 0)) (the ReLU's backward
  // rule), C = round(P + bias[row]), relu_out = max(C, 0); each rounded as
  // the separate operations round.
  const void *bias;
  void *relu_out;
  const void *share_of;
  // f32 products (TF32 kernel): each operand is stored [rows x 2*kp] as
  // [hi | lo] halves; the K loop runs over three kp-long segments
  // (hi.hi, hi.lo, lo.hi) and p.K = 3 * kp.
  int kp;
  // Split K: each tile's K blocks in `ksplit` ranges of `kper` blocks, one
  // work unit each; a unit's raw f32 accumulator goes to
  // partial[range][row][col] and a second kernel sums the ranges in order
  // and applies the epilogue.  ksplit = 1: the epilogue here.
  int ksplit, kper;
  float *partial;
};

// Tile t of the persistent sequence -> (m block, n block), grouped along M
// so that concurrently resident CTAs share B panels in L2.
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int &mb, int &nb) {
  const int GROUP = 8;
  int group_size = GROUP * num_n;
  int group = t / group_size;
  int first = group * GROUP;
  int gm = min(num_m - first, GROUP);
  int r = t - group * group_size;
  mb = first + r % gm;
  nb = r / gm;
}

template <int BN, int STAGES, bool TF32 = false>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, const Params p) {
  constexpr int KE = TF32 ? 32 : BK;  // elements in one 128-byte row of a stage
  constexpr uint32_t A_BYTES = BM * 128, B_BYTES = BN * 128, STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulators
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *tiles = smem;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
  uint64_t *empty = full + STAGES;
  uint64_t *acc_full = empty + STAGES;
  uint64_t *acc_empty = acc_full + 2;
  uint64_t *drain = acc_empty + 2;
  // Epilogue staging for stores to peers: per epilogue warp, 32 rows of 64
  // 16-bit values (128 bytes, padded to 144), after the barrier block.
  uint16_t *epi_stage = reinterpret_cast<uint16_t *>(smem + STAGES * STAGE_BYTES + 256);
  __shared__ uint32_t tmem_base_slot;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (p.M + BM - 1) / BM, num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int S = p.ksplit;
  const int num_units = num_tiles * S;
  const int k_blocks = (p.K + KE - 1) / KE;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], EPI_WARPS * 32);
    }
    mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch(&map_a);
    tma_prefetch(&map_b);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem_base = tmem_base_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t filled = 0, fill_parity = 0;  // per stage: a fill was issued, and its phase parity
      for (int u = blockIdx.x; u < num_units && !abort_flag; u += gridDim.x) {
        const int t = u / S, ks = u - t * S;
        int mb, nb;
        tile_coords(t, num_m, num_n, mb, nb);
        const int m0 = mb * BM, n0 = nb * BN;
        const int kb_lo = ks * p.kper, kb_hi = min(k_blocks, kb_lo + p.kper);
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, &abort_flag, p.wait_ns)) break;
          uint8_t *sa = tiles + stage * STAGE_BYTES;
          uint8_t *sb = sa + A_BYTES;
          mbar_expect_tx(&full[stage], STAGE_BYTES);
          int k0 = kb * KE, kb0 = k0;
          if (TF32) {
            // segment s of three: A half (hi, hi, lo), B half (hi, lo, hi)
            const int seg_blocks = p.kp / KE, sgm = kb / seg_blocks, kk = (kb - sgm * seg_blocks) * KE;
            k0 = kk + (sgm == 2 ? p.kp : 0);
            kb0 = kk + (sgm == 1 ? p.kp : 0);
          }
          if (TF32) {
            tma_load_2d(sa, &map_a, &full[stage], k0, m0);
            tma_load_2d(sb, &map_b, &full[stage], kb0, n0);
          } else {
          if (p.a_mn) {
            tma_load_2d(sa, &map_a, &full[stage], m0, k0);
            tma_load_2d(sa + 64 * BK * 2, &map_a, &full[stage], m0 + 64, k0);
          } else {
            tma_load_2d(sa, &map_a, &full[stage], k0, m0);
          }
          if (p.b_mn) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + j * 64 * BK * 2, &map_b, &full[stage], n0 + 64 * j, k0);
          } else {
            tma_load_2d(sb, &map_b, &full[stage], k0, n0);
          }
          }
          filled |= 1u << stage;
          fill_parity = (fill_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // On an abort, let every copy this thread started land before the CTA
      // exits: the phase a fill completes is the parity it was issued in.
      if (abort_flag) {
        for (int s = 0; s < STAGES; ++s)
          if (filled & (1u << s)) mbar_drain(&full[s], (fill_parity >> s) & 1u);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      // A/B format: F16 0, BF16 1 (kind::f16); TF32 2 (kind::tf32).
      const uint32_t fmt = TF32 ? 2u : uint32_t(p.elem_is_bf16);
      const uint32_t idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | (uint32_t(p.a_mn) << 15) |
                             (uint32_t(p.b_mn) << 16) | (uint32_t(BN >> 3) << 17) | (uint32_t(BM >> 4) << 24);
      // K advance per 16-element MMA step inside a stage: 32 bytes along a
      // K-major row; 16 rows of 128 bytes down an MN-major tile.
      const uint32_t a_step = p.a_mn ? 16 * 128 : 32, b_step = p.b_mn ? 16 * 128 : 32;
      const uint32_t a_lbo = p.a_mn ? 64 * BK * 2 : 16, b_lbo = p.b_mn ? 64 * BK * 2 : 16;
      int stage = 0;
      uint32_t phase = 0;
      int iter = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++iter) {
        const int buf = iter & 1;
        const uint32_t use = uint32_t(iter >> 1);
        const int ks = u - (u / S) * S;
        const int kb_lo = ks * p.kper, kb_hi = min(k_blocks, kb_lo + p.kper);
        // The accumulator must have been drained by the epilogue.
        if (!mbar_wait(&acc_empty[buf], (use & 1u) ^ 1u, &abort_flag, p.wait_ns)) { ok = false; break; }
        fence_after();
        const uint32_t tmem_d = tmem_base + uint32_t(buf * BN);
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&full[stage], phase, &abort_flag, p.wait_ns)) { ok = false; break; }
          fence_after();
          const uint32_t sa = smem_u32(tiles + stage * STAGE_BYTES), sb = sa + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {  // 32 bytes of K per MMA: 16 f16/bf16 or 8 tf32
            uint64_t da = smem_desc(sa + kk * a_step, a_lbo, 1024);
            uint64_t db = smem_desc(sb + kk * b_step, b_lbo, 1024);
            if (TF32) umma_tf32(tmem_d, da, db, idesc, (kb != kb_lo) || kk);
            else umma(tmem_d, da, db, idesc, (kb != kb_lo) || kk);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&acc_full[buf]);
      }
      // Drain: every MMA issued by this thread completes before TMEM is
      // freed, whatever happened.
      umma_commit(drain);
      mbar_drain(drain, 0);
    }
  } else {
    // ---------------- epilogue ----------------
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    int iter = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++iter) {
      const int buf = iter & 1;
      const uint32_t use = uint32_t(iter >> 1);
      if (!mbar_wait(&acc_full[buf], use & 1u, &abort_flag, p.wait_ns)) break;
      fence_after();
      const int t = u / S, ks = u - t * S;
      int mb, nb;
      tile_coords(t, num_m, num_n, mb, nb);
      const int row = mb * BM + q * 32 + lane;
      const int n0 = nb * BN;
      const uint32_t taddr = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(buf * BN);
      if (!TF32 && p.n_peers) {
        // Stores to peers: each 32-row x 64-column piece goes through
        // shared memory, so the warp writes whole 128-byte row segments
        // (four rows per instruction) to C and to every peer's C, rather
        // than 16 bytes per row per lane.  N is a multiple of 8 here.
        constexpr int PITCH = 72;  // 16-bit values per staged row
        uint16_t *stage = epi_stage + q * 32 * PITCH;
#pragma unroll 1
        for (int c2 = 0; c2 < BN / 64; ++c2) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t r[32];
            tmem_ld32(taddr + uint32_t(c2 * 64 + h * 32), r);
            uint4 *dstp = reinterpret_cast<uint4 *>(stage + lane * PITCH + h * 32);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float a = __uint_as_float(r[8 * k + 2 * e]), b = __uint_as_float(r[8 * k + 2 * e + 1]);
                w[e] = p.elem_is_bf16 ? pack2_bf16(a, b) : pack2_f16(a, b);
              }
              dstp[k] = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
          __syncwarp();
          const int col0 = n0 + c2 * 64;
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int rr = it * 4 + (lane >> 3), seg = lane & 7;
            const int grow = mb * BM + q * 32 + rr, gcol = col0 + seg * 8;
            const uint4 val = *reinterpret_cast<const uint4 *>(stage + rr * PITCH + seg * 8);
            if (grow < p.M && gcol < p.N) {
              const size_t off = size_t(grow) * size_t(p.N) + size_t(gcol);
              *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.c) + off) = val;
#pragma unroll
              for (int i = 0; i < MAX_PEERS; ++i)
                if (i < p.n_peers) *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.peer_c[i]) + off) = val;
            }
          }
          __syncwarp();
        }
        fence_before();
        mbar_arrive(&acc_empty[buf]);
        continue;
      }
      if (S > 1) {
        // One K range of a split tile: the raw f32 accumulator.
        float *prow = p.partial + (size_t(ks) * size_t(p.M) + size_t(row)) * size_t(p.N);
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(taddr + uint32_t(c * 32), r);
          const int col0 = n0 + c * 32;
          if (row < p.M && col0 < p.N) {
            if (col0 + 32 <= p.N && (p.N & 3) == 0) {
#pragma unroll
              for (int j = 0; j < 8; ++j)
                *reinterpret_cast<float4 *>(prow + col0 + 4 * j) =
                    make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (col0 + j < p.N) prow[col0 + j] = __uint_as_float(r[j]);
            }
          }
        }
        fence_before();
        mbar_arrive(&acc_empty[buf]);
        continue;
      }
      uint16_t *crow = static_cast<uint16_t *>(p.c) + size_t(row) * size_t(p.N);
      uint16_t *hrow = static_cast<uint16_t *>(p.relu_out) + size_t(row) * size_t(p.N);
      float bias_row = 0.0f;
      if (p.bias && row < p.M) {
        const uint16_t braw = static_cast<const uint16_t *>(p.bias)[row];
        bias_row = p.elem_is_bf16 ? BF16T::load(braw) : F16T::load(braw);
      }
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(taddr + uint32_t(c * 32), r);
        const int col0 = n0 + c * 32;
        if (TF32) {
          if (row < p.M && col0 < p.N) {
            float *frow = static_cast<float *>(p.c) + size_t(row) * size_t(p.N) + col0;
            if (col0 + 32 <= p.N && p.vec_store) {
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                float4 o = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                       __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
                if (p.accumulate) {
                  const float4 old = *reinterpret_cast<const float4 *>(frow + 4 * j);
                  o = make_float4(__fadd_rn(old.x, o.x), __fadd_rn(old.y, o.y), __fadd_rn(old.z, o.z),
                                  __fadd_rn(old.w, o.w));
                }
                *reinterpret_cast<float4 *>(frow + 4 * j) = o;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (col0 + j < p.N) {
                  const float v = __uint_as_float(r[j]);
                  frow[j] = p.accumulate ? __fadd_rn(frow[j], v) : v;
                }
            }
          }
          continue;
        }
        if (row < p.M && col0 < p.N) {
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          const bool whole = col0 + 32 <= p.N && p.vec_store;
          if (p.accumulate) {
            if (whole) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                uint4 old = *reinterpret_cast<const uint4 *>(crow + col0 + 8 * j);
                const uint32_t w[4] = {old.x, old.y, old.z, old.w};
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                  uint16_t lo = uint16_t(w[h] & 0xffffu), hi = uint16_t(w[h] >> 16);
                  float flo = p.elem_is_bf16 ? BF16T::load(lo) : F16T::load(lo);
                  float fhi = p.elem_is_bf16 ? BF16T::load(hi) : F16T::load(hi);
                  v[8 * j + 2 * h] = __fadd_rn(flo, v[8 * j + 2 * h]);
                  v[8 * j + 2 * h + 1] = __fadd_rn(fhi, v[8 * j + 2 * h + 1]);
                }
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (col0 + j < p.N) {
                  uint16_t o = crow[col0 + j];
                  v[j] = __fadd_rn(p.elem_is_bf16 ? BF16T::load(o) : F16T::load(o), v[j]);
                }
              }
            }
          }
          if (p.share_of) {
            // The ReLU's backward rule: round(round(P) * MaxShare(A, 0)).
            const uint16_t *arow = static_cast<const uint16_t *>(p.share_of) + size_t(row) * size_t(p.N) + col0;
            uint16_t araw[32];
            if (whole) {
#pragma unroll
              for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4 *>(araw + 8 * j) = *reinterpret_cast<const uint4 *>(arow + 8 * j);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) araw[j] = col0 + j < p.N ? arow[j] : uint16_t(0);
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float z = p.elem_is_bf16 ? BF16T::load(BF16T::store(v[j])) : F16T::load(F16T::store(v[j]));
              const float a = p.elem_is_bf16 ? BF16T::load(araw[j]) : F16T::load(araw[j]);
              v[j] = __fmul_rn(z, a > 0.0f ? 1.0f : (a < 0.0f ? 0.0f : 0.5f));
            }
          }
          if (p.bias) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float z = p.elem_is_bf16 ? BF16T::load(BF16T::store(v[j])) : F16T::load(F16T::store(v[j]));
              v[j] = __fadd_rn(z, bias_row);
            }
          }
          if (p.relu_out) {
            // max(round(a), 0) is exact in the element type.
            if (whole) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                uint32_t w[4];
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                  const float a = v[8 * j + 2 * h], b = v[8 * j + 2 * h + 1];
                  const float ra = p.elem_is_bf16 ? BF16T::load(BF16T::store(a)) : F16T::load(F16T::store(a));
                  const float rb = p.elem_is_bf16 ? BF16T::load(BF16T::store(b)) : F16T::load(F16T::store(b));
                  w[h] = p.elem_is_bf16 ? pack2_bf16(fmaxf(ra, 0.0f), fmaxf(rb, 0.0f))
                                        : pack2_f16(fmaxf(ra, 0.0f), fmaxf(rb, 0.0f));
                }
                *reinterpret_cast<uint4 *>(hrow + col0 + 8 * j) = make_uint4(w[0], w[1], w[2], w[3]);
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (col0 + j < p.N) {
                  const float ra = p.elem_is_bf16 ? BF16T::load(BF16T::store(v[j])) : F16T::load(F16T::store(v[j]));
                  hrow[col0 + j] = p.elem_is_bf16 ? BF16T::store(fmaxf(ra, 0.0f)) : F16T::store(fmaxf(ra, 0.0f));
                }
            }
          }
          const size_t at = size_t(row) * size_t(p.N) + size_t(col0);
          if (whole) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint32_t w[4];
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                const float a = v[8 * j + 2 * h], b = v[8 * j + 2 * h + 1];
                w[h] = p.elem_is_bf16 ? pack2_bf16(a, b) : pack2_f16(a, b);
              }
              const uint4 q4 = make_uint4(w[0], w[1], w[2], w[3]);
              *reinterpret_cast<uint4 *>(crow + col0 + 8 * j) = q4;
#pragma unroll
              for (int i = 0; i < MAX_PEERS; ++i)
                if (i < p.n_peers) *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.peer_c[i]) + at + 8 * j) = q4;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < p.N) {
                const uint16_t o = p.elem_is_bf16 ? BF16T::store(v[j]) : F16T::store(v[j]);
                crow[col0 + j] = o;
#pragma unroll
                for (int i = 0; i < MAX_PEERS; ++i)
                  if (i < p.n_peers) static_cast<uint16_t *>(p.peer_c[i])[at + j] = o;
              }
          }
        }
      }
      fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
    // Stores to peers are ordered before whatever this GPU does next (the
    // collective that tells the peers the product is complete).
    if (p.n_peers) __threadfence_system();
  }

  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
  }
}

// ---- host: tensor maps -------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// A 2-D map of a row-major [outer, inner] matrix with `box` = {64, box_outer}
// and 128-byte swizzle.
int make_map(CUtensorMap *map, const void *base, bool bf16, uint64_t inner, uint64_t outer, uint32_t box_outer,
             bool f32 = false) {
  auto fn = encode_fn();
  if (!fn) return fail(TC_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  const uint64_t eb = f32 ? 4 : 2;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * eb};
  cuuint32_t box[2] = {cuuint32_t(128 / eb), box_outer};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType type = f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                       : bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, type, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TC_ECUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return TC_OK;
}

// An f32 operand as TF32 halves: row r of `out` (2 * kp floats) is
// [hi(x[r, 0..K)), zeros | lo(x[r, 0..K)), zeros] with hi = tf32(x) (round
// to nearest, ties away) and lo = tf32(x - hi); x[r, k] is src[r*sr + k*sc].
// A 32 x 32 tile through shared memory when the source steps by one along r.
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t u;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(u) : "f"(x));
  return __uint_as_float(u);
}
__global__ void __launch_bounds__(256) split_tf32(const float *src, long long R, long long K, long long sr,
                                                  long long sc, float *out, long long kp) {
  __shared__ float tile[32][33];
  const long long r0 = (long long)blockIdx.y * 32, k0 = (long long)blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  if (sc != 1) {
    // read along r (consecutive threads, consecutive rows), write along k
    for (int i = ty; i < 32; i += 8) {
      const long long k = k0 + i, r = r0 + tx;
      tile[i][tx] = (r < R && k < K) ? __ldg(src + r * sr + k * sc) : 0.0f;
    }
    __syncthreads();
  }
  for (int i = ty; i < 32; i += 8) {
    const long long r = r0 + i, k = k0 + tx;
    if (r >= R) continue;
    const float x = sc != 1 ? tile[tx][i] : (k < K ? __ldg(src + r * sr + k) : 0.0f);
    const float hi = to_tf32(x);
    out[r * 2 * kp + k] = hi;
    out[r * 2 * kp + kp + k] = to_tf32(__fsub_rn(x, hi));
  }
}

template <int BN, int STAGES, bool TF32 = false>
int launch(const CUtensorMap &ma, const CUtensorMap &mb, const Params &p, cudaStream_t stream) {
  // tiles, 1024 bytes of alignment slack, the barriers (256), the epilogue
  // staging (4 warps x 32 rows x 144 bytes)
  constexpr size_t smem = size_t(STAGES) * (BM * 128 + BN * 128) + 1024 + 256 + 4 * 32 * 144;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    if (int st = check_cuda(cudaFuncSetAttribute(gemm_tc<BN, STAGES, TF32>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
                            "cudaFuncSetAttribute"))
      return st;
    configured[dev & 63] = true;
  }
  const int units = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN) * std::max(1, p.ksplit);
  const int grid = std::min(units, std::max(1, sm_count() - reserved_sms()));
  gemm_tc<BN, STAGES, TF32><<<grid, THREADS, smem, stream>>>(ma, mb, p);
  return check_launch("gemm (tcgen05)");
}

// Split K, second pass: the K ranges' f32 accumulators summed in range
// order, then what the GEMM epilogue would have done with the sum.  Four
// adjacent columns per thread when rows are a multiple of four long.
template <class T>
__device__ __forceinline__ float finish_one(float v, typename T::S *c, size_t i, bool accumulate,
                                            const typename T::S *share_of, float bias, bool has_bias,
                                            typename T::S *relu_out) {
  if (accumulate) v = __fadd_rn(T::load(c[i]), v);
  if (share_of) {
    const float a = T::load(share_of[i]);
    v = __fmul_rn(T::load(T::store(v)), a > 0.0f ? 1.0f : (a < 0.0f ? 0.0f : 0.5f));
  }
  if (has_bias) v = __fadd_rn(T::load(T::store(v)), bias);
  if (relu_out) relu_out[i] = T::store(fmaxf(T::load(T::store(v)), 0.0f));
  return v;
}

template <class T>
__global__ void __launch_bounds__(256) splitk_finish(const float *partial, int ranges, long long M, long long N,
                                                     typename T::S *c, bool accumulate, const typename T::S *share_of,
                                                     const typename T::S *bias, typename T::S *relu_out) {
  const long long total = M * N;
  const long long stride = (long long)gridDim.x * blockDim.x;
  if ((N & 3) == 0) {
    for (long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x; q < total / 4; q += stride) {
      const size_t i = size_t(q) * 4;
      float4 v = *reinterpret_cast<const float4 *>(partial + i);
      for (int r = 1; r < ranges; ++r) {
        const float4 w = *reinterpret_cast<const float4 *>(partial + size_t(r) * size_t(total) + i);
        v = make_float4(__fadd_rn(v.x, w.x), __fadd_rn(v.y, w.y), __fadd_rn(v.z, w.z), __fadd_rn(v.w, w.w));
      }
      const float b = bias ? T::load(bias[i / size_t(N)]) : 0.0f;
      const float o[4] = {finish_one<T>(v.x, c, i, accumulate, share_of, b, bias, relu_out),
                          finish_one<T>(v.y, c, i + 1, accumulate, share_of, b, bias, relu_out),
                          finish_one<T>(v.z, c, i + 2, accumulate, share_of, b, bias, relu_out),
                          finish_one<T>(v.w, c, i + 3, accumulate, share_of, b, bias, relu_out)};
      if (sizeof(typename T::S) == 2 && (reinterpret_cast<uintptr_t>(c) & 7u) == 0) {
        // the four results in one 8-byte store
        union { uint2 raw; typename T::S e[4]; } w;
#pragma unroll
        for (int j = 0; j < 4; ++j) w.e[j] = T::store(o[j]);
        *reinterpret_cast<uint2 *>(c + i) = w.raw;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) c[i + j] = T::store(o[j]);
      }
    }
    return;
  }
  for (long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x; q < total; q += stride) {
    const size_t i = size_t(q);
    float v = partial[i];
    for (int r = 1; r < ranges; ++r) v = __fadd_rn(v, partial[size_t(r) * size_t(total) + i]);
    const float b = bias ? T::load(bias[i / size_t(N)]) : 0.0f;
    c[i] = T::store(finish_one<T>(v, c, i, accumulate, share_of, b, bias, relu_out));
  }
}

// Tile width and K split for an M x N product of k_blocks K blocks: 128 x 256
// tiles when they fill the SMs; otherwise split K (2 or 4 ranges of at least
// 16 blocks) while the units still fit in one wave; otherwise 128 x 128 tiles
// when even twice as many of them fit in one wave.
struct Plan {
  int bn, ksplit, kper;
};
Plan plan_tiles(long long M, long long N, int k_blocks, bool may_split) {
  const int sms = sm_count();
  const long long t256 = ((M + BM - 1) / BM) * ((N + 255) / 256);
  if (t256 >= sms) return {256, 1, k_blocks};
  if (may_split)
    for (int cand : {4, 2})
      if (t256 * cand <= sms && k_blocks / cand >= 16) return {256, cand, (k_blocks + cand - 1) / cand};
  if (t256 * 2 <= sms) return {128, 1, k_blocks};
  return {256, 1, k_blocks};
}

template <class T>
int finish_split(const Params &p, const Epilogue &e, cudaStream_t stream) {
  using S = typename T::S;
  const long long total = (long long)p.M * p.N;
  splitk_finish<T><<<grid_for(size_t(total), 256, 8), 256, 0, stream>>>(
      p.partial, p.ksplit, p.M, p.N, static_cast<S *>(p.c), p.accumulate != 0, static_cast<const S *>(e.share_of),
      static_cast<const S *>(e.bias), static_cast<S *>(e.relu_out));
  return check_launch("gemm (split-K finish)");
}

}  // namespace

int gemm_tc_run(int dtype, int transposed, size_t rows, size_t inner, size_t cols, const void *a, const void *b,
                void *c, bool accumulate, cudaStream_t stream) {
  return gemm_tc_run_peers(dtype, transposed, rows, inner, cols, a, b, c, accumulate, nullptr, 0, stream);
}

int gemm_tc_run_peers(int dtype, int transposed, size_t rows, size_t inner, size_t cols, const void *a,
                      const void *b, void *c, bool accumulate, void *const *peer_c, int n_peers,
                      cudaStream_t stream) {
  return gemm_tc_run_full(dtype, transposed, rows, inner, cols, a, b, c, accumulate, peer_c, n_peers, Epilogue{},
                          stream);
}

int gemm_tc_run_full(int dtype, int transposed, size_t rows, size_t inner, size_t cols, const void *a,
                     const void *b, void *c, bool accumulate, void *const *peer_c, int n_peers, const Epilogue &e,
                     cudaStream_t stream) {
  if (n_peers < 0 || n_peers > MAX_PEERS) return fail(TC_EINVAL, "gemm: %d peers, at most %d", n_peers, MAX_PEERS);
  if ((e.bias || e.relu_out || e.share_of) && (accumulate || n_peers))
    return fail(TC_EINVAL, "gemm: an epilogue neither accumulates nor stores to peers");
  if (dtype != TC_BF16 && dtype != TC_F16) return TC_ENOTSUP;
  if (inner < 16 || rows > 0x7fffffffu || cols > 0x7fffffffu || inner > 0x7fffffffu) return TC_ENOTSUP;
  const bool a_mn = transposed == TC_TRANS_LEFT;   // A stored [K, M]
  const bool b_mn = transposed != TC_TRANS_RIGHT;  // B stored [K, N]
  // TMA: 16-byte aligned bases and row pitches.
  const uint64_t a_inner = a_mn ? rows : inner, b_inner = b_mn ? cols : inner;
  if ((uintptr_t(a) & 15u) || (uintptr_t(b) & 15u) || (a_inner * 2) % 16 || (b_inner * 2) % 16) return TC_ENOTSUP;
  const bool bf16 = dtype == TC_BF16;
  Params p{};
  p.wait_ns = g_wait_ns.load();
  p.M = int(rows);
  p.N = int(cols);
  p.K = int(inner);
  p.a_mn = a_mn;
  p.b_mn = b_mn;
  p.accumulate = accumulate;
  p.c = c;
  p.elem_is_bf16 = bf16;
  p.vec_store = (uintptr_t(c) & 15u) == 0 && (cols * 2) % 16 == 0;
  p.bias = e.bias;
  p.relu_out = e.relu_out;
  p.share_of = e.share_of;
  if (e.relu_out && (uintptr_t(e.relu_out) & 15u)) p.vec_store = 0;
  if (e.share_of && (uintptr_t(e.share_of) & 15u)) p.vec_store = 0;
  p.n_peers = n_peers;
  for (int i = 0; i < MAX_PEERS; ++i) {
    p.peer_c[i] = i < n_peers ? peer_c[i] : nullptr;
    if (i < n_peers && (uintptr_t(peer_c[i]) & 15u)) p.vec_store = 0;
  }
  // The peer epilogue stores 16-byte segments: rows of C 16-byte aligned.
  if (n_peers && (!p.vec_store || cols % 8)) return TC_ENOTSUP;
  const int k_blocks = int((inner + BK - 1) / BK);
  const Plan pl = plan_tiles((long long)rows, (long long)cols, k_blocks, n_peers == 0);
  const int BN = pl.bn;
  p.ksplit = pl.ksplit;
  p.kper = pl.kper;
  p.partial = nullptr;
  if (p.ksplit > 1) {
    void *w = nullptr;
    if (int st = scratch(size_t(p.ksplit) * rows * cols * sizeof(float), &w, stream)) return st;
    p.partial = static_cast<float *>(w);
  }
  CUtensorMap ma, mb;
  if (int st = a_mn ? make_map(&ma, a, bf16, rows, inner, BK) : make_map(&ma, a, bf16, inner, rows, BM)) return st;
  if (int st = b_mn ? make_map(&mb, b, bf16, cols, inner, BK) : make_map(&mb, b, bf16, inner, cols, BN)) return st;
  if (int st = BN == 256 ? launch<256, 4>(ma, mb, p, stream) : launch<128, 6>(ma, mb, p, stream)) return st;
  if (p.ksplit == 1) return TC_OK;
  return bf16 ? finish_split<BF16T>(p, e, stream) : finish_split<F16T>(p, e, stream);
}

int gemm_tf32_run(int transposed, size_t rows, size_t inner, size_t cols, const void *a, const void *b, void *c,
                  bool accumulate, cudaStream_t stream) {
  if (rows > 0x7fffffffu || cols > 0x7fffffffu || inner > 0x2aaaaaa0u) return TC_ENOTSUP;
  const long long kp = ((long long)inner + 31) / 32 * 32;
  const Plan pl = plan_tiles((long long)rows, (long long)cols, int(3 * kp / 32), true);
  const size_t operand_floats = size_t(rows + cols) * size_t(2 * kp);
  const size_t partial_floats = pl.ksplit > 1 ? size_t(pl.ksplit) * rows * cols : 0;
  void *scratch_p = nullptr;
  if (int st = scratch((operand_floats + partial_floats) * sizeof(float), &scratch_p, stream)) return st;
  float *ah = static_cast<float *>(scratch_p), *bh = ah + size_t(rows) * size_t(2 * kp);
  // A as [rows x K]: element (m, k); B as [cols x K]: element (n, k).
  const long long a_sr = transposed == TC_TRANS_LEFT ? 1 : (long long)inner;
  const long long a_sc = transposed == TC_TRANS_LEFT ? (long long)rows : 1;
  const long long b_sr = transposed == TC_TRANS_RIGHT ? (long long)inner : 1;
  const long long b_sc = transposed == TC_TRANS_RIGHT ? 1 : (long long)cols;
  dim3 ga(unsigned(kp / 32), unsigned((rows + 31) / 32)), gb(unsigned(kp / 32), unsigned((cols + 31) / 32));
  split_tf32<<<ga, 256, 0, stream>>>(static_cast<const float *>(a), (long long)rows, (long long)inner, a_sr, a_sc, ah,
                                     kp);
  split_tf32<<<gb, 256, 0, stream>>>(static_cast<const float *>(b), (long long)cols, (long long)inner, b_sr, b_sc, bh,
                                     kp);
  if (int st = check_launch("gemm (tf32 split)")) return st;
  Params p{};
  p.wait_ns = g_wait_ns.load();
  p.M = int(rows);
  p.N = int(cols);
  p.K = int(3 * kp);
  p.kp = int(kp);
  p.a_mn = 0;
  p.b_mn = 0;
  p.accumulate = accumulate;
  p.c = c;
  p.vec_store = (uintptr_t(c) & 15u) == 0 && cols % 4 == 0;
  const int BN = pl.bn;
  p.ksplit = pl.ksplit;
  p.kper = pl.kper;
  p.partial = pl.ksplit > 1 ? ah + operand_floats : nullptr;
  CUtensorMap ma, mb;
  if (int st = make_map(&ma, ah, false, uint64_t(2 * kp), rows, BM, true)) return st;
  if (int st = make_map(&mb, bh, false, uint64_t(2 * kp), cols, BN, true)) return st;
  if (int st = BN == 256 ? launch<256, 4, true>(ma, mb, p, stream) : launch<128, 6, true>(ma, mb, p, stream))
    return st;
  if (p.ksplit == 1) return TC_OK;
  return finish_split<F32T>(p, Epilogue{}, stream);
}

}  // namespace tc

namespace tc {
int peer_wait_fault();
int peer_wait_fault_reset();
void set_peer_wait_limit(unsigned long long ns);
}

// How long the tensor-core GEMM's pipeline waits last before a CTA gives up
// (default 2 s); 0 restores the default.  For tests of the failure path.
extern "C" int tc_set_wait_limit(unsigned long long ns) {
  tc::g_wait_ns.store(ns ? ns : 2000000000ull);
  return TC_OK;
}

// How long a data-parallel step waits for another rank's flag (default 5
// s); 0 restores the default.  For tests of the failure path.
extern "C" int tc_set_peer_wait_limit(unsigned long long ns) {
  tc::set_peer_wait_limit(ns);
  return TC_OK;
}

// Clear the records of waits that gave up.
extern "C" int tc_device_status_reset(void) {
  const int zero = 0;
  if (int st = tc::check_cuda(cudaMemcpyToSymbol(tc::g_gemm_fault, &zero, sizeof(int)), "cudaMemcpyToSymbol"))
    return st;
  return tc::peer_wait_fault_reset();
}

extern "C" int tc_device_status(int *fault) {
  int h = 0;
  if (int st = tc::check_cuda(cudaMemcpyFromSymbol(&h, tc::g_gemm_fault, sizeof(int)), "cudaMemcpyFromSymbol"))
    return st;
  const int peer = tc::peer_wait_fault();
  if (fault) *fault = h || peer;
  if (h) return tc::fail(TC_ETIMEOUT, "a tensor-core GEMM gave up waiting on its pipeline");
  if (peer) return tc::fail(TC_ETIMEOUT, "a wait for another rank's flag gave up");
  return TC_OK;
}
