// gemm_tn.cu -- persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   C[M][N] (bf16, row-major) = alpha * A[M][K] (row-major) . B (column-major, [N][K])
//
// Replaces the reference's single-tile MMA issue loops
// (umma_throughput/umma_tput.cu:491-522, tcgen05_sparse_mma/tcgen05_sparse_mma.cu:490-516),
// which re-issue tcgen05.mma on one fixed SMEM tile and never read D back, with
// a complete GEMM:
//
//   warp 0      TMA producer: 2D tiled loads (128B swizzle, K-major) of A and B
//               into a STAGES-deep shared-memory ring; full/empty mbarrier pairs.
//   warp 1      TMEM allocator + MMA issuer: tcgen05.mma.cta_group::CG into an
//               fp32 accumulator in TMEM (two buffers, or one with M_SUB = 2);
//               tcgen05.commit releases ring slots and publishes finished
//               accumulators.
//   Both issuing roles run as whole, converged warps: every lane walks the
//   schedule and waits on the barriers, and one elected lane issues.  The MMA
//   warp does not even branch around an issue: all lanes execute each tcgen05
//   instruction's asm, predicated on the elected lane.
//   warps 2..    epilogue: tcgen05.ld, alpha, fp32 -> bf16, 16-byte vector stores
//               of C.  Four warps (one per TMEM lane quarter) stream 32-column
//               chunks out of a double-buffered accumulator; with one buffer
//               (M_SUB = 2) eight warps (two per quarter, one per column half)
//               read the tile into registers first and release TMEM before
//               storing.
//
// CG = 2 pairs two SMs of a cluster on one 256-row tile: each CTA TMA-loads its
// own 128 rows of A and its own half of the tile's B columns into its own SMEM
// (no multicast); the even CTA issues the pair MMA, whose commit is delivered
// to both CTAs' barriers.  The accumulator of rows [128*rank, 128*rank+128) of
// the pair tile lives in each CTA's own TMEM.
//
// SPARSE (2:4 structured-sparse A, bf16, tcgen05.mma.sp kind::f16): a ring slot
// holds 128 dense K (two 128-byte swizzle atoms of B, one atom of the compressed
// A) and the slot's metadata block (128 lanes x 16 bytes, the engine's
// TMEM-ready layout, see meta_ready_kernel in datagen.cu).  The MMA thread moves
// the metadata block into a 4-deep ring of TMEM columns with tcgen05.cp
// (ordered before its MMAs) and issues 4 sparse MMAs of dense K = 32.
//
// Block-scaled (NVFP4: e2m1 + ue4m3 per 16, kind::mxf4nvf4.block_scale.block16;
// MXFP8: e4m3 + E8M0 per 32, kind::mxf8f6f4.block_scale; MXFP4: e2m1 + E8M0 per
// 32, kind::mxf4.block_scale.block32): a ring slot holds 128 bytes of K of A and
// B plus the slot's scale factors, laid out by sf_ready_kernel (datagen.cu) as
// 512-byte blocks of 32 rows x 16 bytes, one per 4-byte group of scales (a group
// is one NVFP4 MMA, four MXFP8 MMAs or two MXFP4 MMAs).  Per group the MMA thread
// copies SFA (this CTA's 128 rows, 4 columns) and SFB (the tile's N rows padded
// to 256, 8 columns) into TMEM with tcgen05.cp.32x128b.warpx4, which replicates
// the 32 rows into the four lane quarters as the 4x1 scale-factor data path
// expects; each MMA picks its byte of the group with the scale-factor ids.  With
// cta_group::2 each CTA stages its own SFA and the full SFB, and the leader's
// copies fill both CTAs' TMEM.
//
// M_SUB = 2 (sparse, block-scaled): each CTA holds two 128-row sub-tiles of A against one B
// tile and issues two MMAs per K step into two accumulators (columns [0, BN) and
// [BN, 2 BN)).  B then costs half the SMEM fill bytes per MMA, which is what the
// sparse path is short of (at the 2x sparse MMA rate a 256 x 224 pair tile needs
// about 100 B/cycle per SM of L2 -> SMEM traffic, a 512 x 224 one about 69).
// The 2 x 224 accumulator columns leave no room for a second TMEM buffer; the
// epilogue holds TMEM only while it reads the accumulator into registers and
// stores C while the next tile's MMAs run.
//
// Tiles are visited by a static persistent schedule (tile = cluster id + i *
// clusters) in a grouped raster order for L2 reuse.  Every wait is bounded.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <atomic>

#include "b2g_desc.h"
#include "b2g_gemm.h"
#include "b2g_ptx.cuh"

namespace b2g {

// Epilogue warps: 4 (one per TMEM lane quarter) when the accumulator is double
// buffered; 8 (two per quarter, one per column half) with one buffer (M_SUB = 2)
__host__ __device__ constexpr int epi_warps(int m_sub) { return m_sub == 2 ? 8 : 4; }
__host__ __device__ constexpr int kernel_threads(int m_sub) { return 64 + 32 * epi_warps(m_sub); }
// 16-column chunks of one epilogue warp's column half: BN <= 256; with two
// sub-tiles BN <= 224 when side operands share TMEM with the accumulators (sparse
// metadata, scale factors), BN <= 256 for dense (2 x 256 accumulator columns fill TMEM)
__host__ __device__ constexpr int epi_chunks(int m_sub, int var) {
  return m_sub == 2 ? (var == GEMM_DENSE ? 8 : 7) : 8;
}
constexpr int kRowsPerCta = 128;     // A rows per CTA == TMEM lanes
constexpr int kKBytes = 128;         // K extent of one A ring slot, in bytes (one 128B swizzle atom)
constexpr int kMmaKBytes = 32;       // A bytes of K consumed by one tcgen05.mma
constexpr int kMaxStages = 8;
constexpr int kMetaRing = 4;         // metadata blocks resident in TMEM
// (the side operands' tensor maps view their buffers in kSideLine-byte lines: b2g_gemm.h)
// 2:4 metadata of one ring slot and 128-row sub-tile: one bit per dense K element
// and row.  kind::f16: 128 dense K, 4 TMEM columns (128 lanes x 16 bytes);
// kind::f8f6f4 / kind::i8: 256 dense K, 8 columns (two such 2 KB halves).
__host__ __device__ constexpr int meta_cols(int kind) {
  // (kind::mxf4: 4:8 in pairs of packed e2m1 is 2:4 on bytes, the 8-bit layout)
  return (kind == KIND_F8F6F4 || kind == KIND_I8 || kind == KIND_MXF8F6F4 || kind == KIND_MXF4 ||
          kind == KIND_MXF4NVF4)
             ? 8
             : 4;
}
__host__ __device__ constexpr int meta_slot_bytes(int kind) { return meta_cols(kind) * 512; }
// Block-scaled side operands per ring slot: SFA one 512-byte block (32 rows x 16 B)
// per scale group and 128-row sub-tile, SFB two (256 rows) per group.
__host__ __device__ constexpr int sfa_bytes(int var) { return gemm_sf_groups(var) * 512; }
__host__ __device__ constexpr int sfb_bytes(int var) { return gemm_sf_groups(var) * 1024; }
// TMEM columns of one slot's scale factors: per MMA SFA 4 per A sub-tile + SFB 8
__host__ __device__ constexpr int sf_cols_per_slot(int var, int m_sub) {
  return gemm_sf_groups(var) * (4 * m_sub + 8);
}
// One TMEM region for the scale factors of the current slot: tcgen05.cp and
// tcgen05.mma issued by the same thread execute in order, so the copy for slot
// s+1 cannot overwrite scale factors that slot s's MMAs still read.
constexpr int kSfRing = 1;

constexpr int VAR_DENSE = GEMM_DENSE, VAR_SPARSE = GEMM_SPARSE, VAR_NVFP4 = GEMM_NVFP4;

struct SmemCarve {
  // offsets from the 1024-aligned dynamic smem base
  uint32_t a, b, meta, bars, tmem_slot, abort_flag, total;
};

// per-slot bytes of the side operands: metadata, then scale factors (SFA per
// sub-tile, SFB)
__host__ __device__ inline int side_bytes(int var, int m_sub, int kind) {
  return (gemm_sparse(var) ? m_sub * meta_slot_bytes(kind) : 0) +
         (gemm_block_scaled(var) ? m_sub * sfa_bytes(var) + sfb_bytes(var) : 0);
}

// ka: 128-byte K atoms per ring slot (2 for the dense small-N instances)
__host__ __device__ inline SmemCarve carve(int stages, int b_rows, int var, int m_sub, int ka,
                                           int kind) {
  SmemCarve c;
  c.a = 0;
  c.b = c.a + stages * ka * m_sub * kRowsPerCta * kKBytes;
  c.meta = c.b + stages * (gemm_sparse(var) ? 2 : ka) * b_rows * kKBytes;
  c.bars = c.meta + stages * side_bytes(var, m_sub, kind);
  c.tmem_slot = c.bars + (2 * kMaxStages + 4 + 1) * 8;
  c.abort_flag = c.tmem_slot + 4;
  c.total = c.abort_flag + 4;
  return c;
}

// TS operand mode: one slot's A (128 lanes x 128 bytes) in TMEM, reused every
// slot like the scale factors (copy and MMA execute in issue order).
constexpr int kTsACols = 32;

// accumulator buffers in TMEM: two (the epilogue of tile i overlaps the MMAs of
// tile i+1) unless two sub-tiles' accumulators fill TMEM
__host__ __device__ constexpr int acc_buffers(int m_sub) { return m_sub == 2 ? 1 : 2; }

__host__ __device__ inline uint32_t tmem_columns(int tile_n, int var, bool ts, int m_sub, int kind) {
  const uint32_t need = (uint32_t)(acc_buffers(m_sub) * m_sub * tile_n) +
                        (gemm_sparse(var) ? (uint32_t)(meta_cols(kind) * kMetaRing * m_sub) : 0u) +
                        (gemm_block_scaled(var) ? (uint32_t)(sf_cols_per_slot(var, m_sub) * kSfRing) : 0u) +
                        (ts ? (uint32_t)kTsACols : 0u);
  uint32_t c = 32;
  while (c < need) c <<= 1;
  return c;
}

__device__ __forceinline__ void tile_coords(int t, int num_m_tiles, int num_n_tiles, int group_m,
                                            int& mt, int& nt) {
  const int per_group = group_m * num_n_tiles;
  const int g = t / per_group;
  const int first_m = g * group_m;
  const int gm = min(num_m_tiles - first_m, group_m);
  const int r = t - g * per_group;
  mt = first_m + r % gm;
  nt = r / gm;
}

// One work unit of the persistent schedule: a whole tile, or one K range of a
// tile of the split tail.
struct Unit {
  int tile;      // tile index in raster order
  int kb0, kb1;  // ring slots [kb0, kb1) of K
  int split;     // 0 for whole tiles and for the split that finishes a tail tile
  int vt;        // tail tile index (tile - tail_start), -1 for whole tiles
};

__host__ __device__ inline int num_units(const GemmArgs& a, int num_tiles) {
  return a.tail_split > 1 ? a.tail_start + (num_tiles - a.tail_start) * a.tail_split : num_tiles;
}

__device__ __forceinline__ Unit unit_of(int u, const GemmArgs& a) {
  Unit w;
  if (a.tail_split <= 1 || u < a.tail_start) {
    w.tile = u;
    w.kb0 = 0;
    w.kb1 = a.k_blocks;
    w.split = 0;
    w.vt = -1;
  } else {
    const int v = u - a.tail_start;
    w.vt = v / a.tail_split;
    w.split = v - w.vt * a.tail_split;
    w.tile = a.tail_start + w.vt;
    w.kb0 = (int)((int64_t)w.split * a.k_blocks / a.tail_split);
    w.kb1 = (int)((int64_t)(w.split + 1) * a.k_blocks / a.tail_split);
  }
  return w;
}

// Bounded wait for a split-tail flag to carry this launch's stamp (one lane).
__device__ __forceinline__ bool wait_stamp(const uint32_t* f, uint32_t want, volatile int* abort,
                                           uint32_t* err, uint64_t limit_ns) {
  return flag_wait(f, want, abort, err, ERRW_TIMEOUT_EPILOGUE, limit_ns);
}

// KA: 128-byte K atoms per ring slot.  KA = 2 (dense SS, one sub-tile) halves the
// per-slot barrier, fence and commit costs per MMA for tiles whose MMAs are short.
// WS: the MMAs are the weight-stationary form tcgen05.mma.ws{.sp} (cta_group::1,
// 128-row tiles, tile_n 64 / 128 / 256; its M = 128 accumulator has the layout of
// the ordinary cta_group::1 MMA, so the epilogue is shared).
template <int KIND, int CG, int VAR, bool TS, int MS, int KA = 1, bool WS = false>
__global__ void __launch_bounds__(kernel_threads(MS), 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmE, const __grid_constant__ CUtensorMap tmF,
                   const __grid_constant__ CUtensorMap tmG, const GemmArgs args) {
  constexpr bool SPARSE = gemm_sparse(VAR);
  constexpr bool NVFP4 = gemm_block_scaled(VAR);  // any block-scaled kind
  constexpr int SFG = gemm_sf_groups(VAR);         // scale groups per ring slot
  constexpr int MPG = 4 / SFG;                     // MMAs per scale group
  static_assert(!TS || VAR == VAR_DENSE, "TS operands are built for the dense variant");
  static_assert(MS == 1 || (MS == 2 && !TS), "two sub-tiles: SS operands only");
  constexpr int ACC = acc_buffers(MS);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int BN = args.tile_n;           // N extent of the MMA (whole pair for CG = 2)
  const int b_rows = BN / CG;           // B rows (N columns) held by this CTA
  const int stages = args.stages;
  static_assert(KA == 1 || (VAR == VAR_DENSE && !TS && MS == 1), "two K atoms: dense SS only");
  static_assert(!WS || (CG == 1 && !TS && MS == 1 && KA == 1 && KIND <= 3 &&
                        (VAR == VAR_DENSE || VAR == VAR_SPARSE)),
                ".ws: cta_group::1, SS, one sub-tile, dense or sparse tf32 / f16 / f8f6f4 / i8");
  const SmemCarve sc = carve(stages, b_rows, VAR, MS, KA, KIND);
  constexpr int MCOLS = meta_cols(KIND);          // sparse: metadata columns per slot, sub-tile
  constexpr int MBYTES = meta_slot_bytes(KIND);   // and its bytes in shared memory

  const uint32_t base = smem_u32(smem);
  const uint32_t sA = base + sc.a;
  const uint32_t sB = base + sc.b;
  const uint32_t sE = base + sc.meta;
  const uint32_t bar_full = base + sc.bars;                  // [stages]
  const uint32_t bar_empty = bar_full + kMaxStages * 8;      // [stages]
  const uint32_t bar_tfull = bar_empty + kMaxStages * 8;     // [2]
  const uint32_t bar_tempty = bar_tfull + 2 * 8;             // [2]
  const uint32_t bar_drain = bar_tempty + 2 * 8;             // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + sc.tmem_slot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + sc.abort_flag);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = (CG == 2) ? cluster_ctarank() : 0u;
  const bool leader = (rank == 0);
  const uint32_t a_bytes = kRowsPerCta * kKBytes;            // one 128-row A sub-tile
  const uint32_t a_slot = KA * MS * a_bytes;                 // A bytes per ring slot
  const uint32_t b_bytes = b_rows * kKBytes;                 // one 128-byte K atom of B
  const uint32_t b_slot = (SPARSE ? 2 : KA) * b_bytes;       // B bytes per ring slot
  // bytes the slot's copies complete on its barrier: the unpacking loads of fp4 /
  // fp6 count the packed bytes they read (half or three quarters of what they write)
  const uint32_t ab_tx =
      (args.tx_a_bits ? a_slot * (uint32_t)args.tx_a_bits / 8u : a_slot) +
      (args.tx_b_bits ? b_slot * (uint32_t)args.tx_b_bits / 8u : b_slot);
  const uint32_t slot_bytes = ab_tx + side_bytes(VAR, MS, KIND);
  const uint32_t tmem_cols = tmem_columns(BN, VAR, TS, MS, KIND);
  constexpr int kRowsPerTile = kRowsPerCta * MS * CG;        // A rows of one (pair) tile

  uint32_t* trace = args.trace ? args.trace + (size_t)blockIdx.x * kTraceWords : nullptr;
  if (threadIdx.x == 0) {
    trace_store(trace, TR_STAGE, 1);
    for (int s = 0; s < stages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_tfull + 8 * i, 1);
      mbar_init(bar_tempty + 8 * i, epi_warps(MS) * CG);
    }
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (SPARSE || NVFP4) tma_prefetch_desc(&tmE);
    if (NVFP4) tma_prefetch_desc(&tmF);
    if (SPARSE && NVFP4) tma_prefetch_desc(&tmG);
  }
  if (warp == 1) {
    tmem_alloc<CG>(smem_u32(tmem_slot), tmem_cols);
    tmem_relinquish<CG>();
    if (lane == 0) trace_store(trace, TR_STAGE, 2);
  }
  tc_fence_before();
  __syncthreads();
  if (CG == 2) cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) {
    trace_store(trace, TR_TMEM_BASE, tmem_base);
    trace_store(trace, TR_STAGE, 3);
  }

  const int num_tiles = args.num_m_tiles * args.num_n_tiles;
  const int n_units = num_units(args, num_tiles);
  const int cluster_id = blockIdx.x / CG;
  const int num_clusters = gridDim.x / CG;
  const int k_blocks = args.k_blocks;
  // Tensor-map x units per ring slot: A's atom holds 128 bytes of stored A (for
  // SPARSE 64 compressed = 128 dense bf16 elements, with B holding two atoms).
  // The packed-e2m1 maps of NVFP4 count bytes, the others count elements.
  const int a_elems_per_kblock = args.elem_bits == 4 ? kKBytes : kKBytes * 8 / args.elem_bits;
  const int b_elems_per_atom = a_elems_per_kblock;
  uint32_t* err = args.err;

  // Role dispatch is by whole warps: a lane-level condition here would send the
  // idle lanes of a role warp into another role's warp-collective code.
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // The whole warp walks the schedule and waits on the ring, so that every
    // address and loop decision stays warp-uniform; the elected lane issues the
    // copies.  (The same loop run by lane 0 alone, the rest of the warp parked,
    // measured about 80 cycles per TMA issue and 650 per ring slot.)
    {
      const bool issuer = elect_one();
      // L2 priority: in the raster order an A row panel is read again by every tile
      // column of its group, wave after wave, while a B column panel is read by the
      // group's tile rows within one wave.  Keeping A (and its metadata / scale
      // factors) resident measured +9 % on the 2:4 sparse cfg3 (B 256 MiB > L2)
      // and +0.5-1 % on the dense shapes against the opposite choice.
      const uint64_t pol_a = l2_policy_evict_last();
      const uint64_t pol_b = l2_policy_evict_normal();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t n_issued = 0;
      for (int u = cluster_id; ok && u < n_units; u += num_clusters) {
        const Unit w = unit_of(u, args);
        int mt, nt;
        tile_coords(w.tile, args.num_m_tiles, args.num_n_tiles, args.group_m, mt, nt);
        const int a_row = mt * kRowsPerTile + (int)rank * kRowsPerCta * MS;
        const int b_row = nt * BN + (int)rank * b_rows;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          const bool got = mbar_wait(bar_empty + 8 * stage, phase ^ 1u, abort_flag, err,
                                     ERRW_TIMEOUT_PRODUCER, args.wait_ns);
          if (!__all_sync(0xffffffffu, got)) {
            if (issuer) trace_store(trace, TR_TIMEOUTS, 1);
            ok = false;
            break;
          }
          const uint32_t fb = (CG == 2) ? mapa_shared(bar_full + 8 * stage, 0) : bar_full + 8 * stage;
          const uint32_t dA = sA + stage * a_slot;
          const uint32_t dB = sB + stage * b_slot;
          const int ka = kb * KA * a_elems_per_kblock;
          const int kbx = kb * (SPARSE ? 2 : KA) * b_elems_per_atom;
          if (issuer) {
            // one 2D tile into this CTA's shared memory; a pair's loads complete on
            // the even CTA's barrier (cta_group::2 form, no multicast)
            auto load = [&](uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t pol) {
              if (CG == 1) tma_load_2d(dst, map, x, y, fb, pol);
              else tma_load_2d_pair(dst, map, x, y, fb, pol);
            };
            if (CG == 1) mbar_arrive_expect_tx(bar_full + 8 * stage, slot_bytes);
            else if (leader) mbar_arrive_expect_tx(bar_full + 8 * stage, CG * slot_bytes);
#pragma unroll
            for (int t = 0; t < KA; ++t) {  // K atom t of the slot: A sub-tiles, then B
#pragma unroll
              for (int sub = 0; sub < MS; ++sub)
                load(dA + (t * MS + sub) * a_bytes, &tmA, ka + t * a_elems_per_kblock,
                     a_row + sub * kRowsPerCta, pol_a);
              load(dB + t * b_bytes, &tmB, kbx + t * b_elems_per_atom, b_row, pol_b);
            }
            if (SPARSE) {
              load(dB + b_bytes, &tmB, kbx + b_elems_per_atom, b_row, pol_b);
#pragma unroll
              for (int sub = 0; sub < MS; ++sub)
                load(sE + stage * side_bytes(VAR, MS, KIND) + sub * MBYTES, &tmE, 0,
                     ((a_row / kRowsPerCta + sub) * k_blocks + kb) * (MBYTES / kSideLine), pol_a);
            }
            if (NVFP4) {
              // scale-factor blocks: [row block][K slot] x (SFA per sub-tile | SFB),
              // after the slot's metadata when A is also sparse
              const uint32_t dS =
                  sE + stage * side_bytes(VAR, MS, KIND) + (SPARSE ? MS * MBYTES : 0);
              const CUtensorMap* map_sfa = SPARSE ? &tmF : &tmE;
              const CUtensorMap* map_sfb = SPARSE ? &tmG : &tmF;
#pragma unroll
              for (int sub = 0; sub < MS; ++sub)
                load(dS + sub * sfa_bytes(VAR), map_sfa, 0,
                     ((a_row / kRowsPerCta + sub) * k_blocks + kb) * (sfa_bytes(VAR) / kSideLine),
                     pol_a);
              load(dS + MS * sfa_bytes(VAR), map_sfb, 0,
                   (nt * k_blocks + kb) * (sfb_bytes(VAR) / kSideLine), pol_b);
            }
          }
          ++n_issued;
          if (issuer) trace_store(trace, TR_TMA_ISSUED, n_issued);
          if (++stage == stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // let in-flight copies land before this CTA can exit
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 200000ull) __nanosleep(1000);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Whole warp, like the producer: the elected lane issues every tcgen05.cp,
    // tcgen05.mma and tcgen05.commit (a commit tracks its own thread's MMAs),
    // through predicated asm that all 32 lanes execute.  Measured per 128-byte K
    // slot of one CTA: lane 0 alone 557 cycles (66 per MMA issue); whole warp with
    // the issues in an elected branch 500; predicated, no branch, about 375 at
    // N = 128 (MMAs 256), i.e. 1.5x the one-lane loop.
    if (leader) {
      const uint32_t on = elect_one() ? 1u : 0u;  // this lane issues
      const bool issuer = on != 0u;
      const uint32_t idesc = args.idesc;
      // side-operand columns follow the accumulators (4-column aligned)
      const uint32_t meta_col0 = tmem_base + (uint32_t)(ACC * MS * BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      uint32_t meta_slot = 0;
      bool ok = true;
      uint32_t n_full = 0, n_tiles = 0;
      for (int u = cluster_id; ok && u < n_units; u += num_clusters) {
        const Unit w = unit_of(u, args);
        const bool got_acc = mbar_wait(bar_tempty + 8 * acc, acc_phase ^ 1u, abort_flag, err,
                                       ERRW_TIMEOUT_MMA, args.wait_ns);
        if (!__all_sync(0xffffffffu, got_acc)) {
          if (issuer) trace_store(trace, TR_TIMEOUTS, 4);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * MS * BN);
        // Unrolled by two: the loop-back work falls on two slots (cfg2 e4m3 8192³ +1.1 %,
        // interleaved: 2997-3008 against 2958-2974 TFLOP/s).
        #pragma unroll 2
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          // the first MMA of a unit overwrites the accumulator
          const uint32_t kfirst = (uint32_t)(kb - w.kb0);
          const bool got = mbar_wait(bar_full + 8 * stage, phase, abort_flag, err,
                                     ERRW_TIMEOUT_MMA, args.wait_ns);
          if (!__all_sync(0xffffffffu, got)) {
            if (issuer) trace_store(trace, TR_TIMEOUTS, 2);
            ok = false;
            break;
          }
          ++n_full;
          tc_fence_after();
          const uint32_t a0 = sA + stage * a_slot;
          const uint32_t b0 = sB + stage * b_slot;
          if constexpr (SPARSE && NVFP4) {
            // Sparse A on a block-scaled kind (2:4 on kind::mxf8f6f4, 4:8 in pairs of
            // packed e2m1 on kind::mxf4): the slot's metadata (8-bit layout: MMA kk reads
            // columns 2 kk, 2 kk + 1) into the metadata ring, then per scale group the
            // SFA / SFB copies and the group's MMAs.  A sparse MMA reads as many scale
            // bytes per row as the dense MMA of its kind, each over twice the dense K:
            // mxf8f6f4 one per 64 K (one group, MMA kk on byte kk), mxf4 two per 128 K
            // (two groups, two MMAs each on bytes 0-1 and 2-3), mxf4nvf4 block16 four
            // per 128 K (four groups, one MMA each)
            const uint32_t e_tmem = meta_col0 + (uint32_t)(MCOLS * MS) * meta_slot;
            const uint32_t dM = sE + stage * side_bytes(VAR, MS, KIND);
#pragma unroll
            for (int sub = 0; sub < MS; ++sub)
#pragma unroll
              for (int hf = 0; hf < MCOLS / 4; ++hf)
                tc_cp_128x128b<CG>(e_tmem + (uint32_t)(MCOLS * sub + 4 * hf),
                                   encode_smem_desc(dM + sub * MBYTES + 2048 * hf, 16, 128, SWZ_NONE),
                                   on);
            const uint32_t dS = dM + MS * MBYTES;
            const uint32_t dSfb = dS + MS * sfa_bytes(VAR);
            const uint32_t sf0 = meta_col0 + (uint32_t)(MCOLS * MS * kMetaRing);
#pragma unroll 1
            for (int g = 0; g < SFG; ++g) {
              const uint32_t sfa0 = sf0 + (uint32_t)(sf_cols_per_slot(VAR, MS) / SFG) * g;
              const uint32_t sfb = sfa0 + 4u * MS;
              tc_cp_32x128b_warpx4<CG>(sfb, encode_smem_desc(dSfb + 1024 * g, 16, 128, SWZ_NONE),
                                       on);
              tc_cp_32x128b_warpx4<CG>(
                  sfb + 4u, encode_smem_desc(dSfb + 1024 * g + 512, 16, 128, SWZ_NONE), on);
#pragma unroll
              for (int sub = 0; sub < MS; ++sub)
                tc_cp_32x128b_warpx4<CG>(
                    sfa0 + 4u * sub,
                    encode_smem_desc(dS + sub * sfa_bytes(VAR) + 512 * g, 16, 128, SWZ_NONE), on);
#pragma unroll
              for (int m = 0; m < MPG; ++m) {
                const int kk = g * MPG + m;
                const uint32_t sf_id = (uint32_t)(m * SFG);
                const uint32_t id_k = idesc | (sf_id << 29) | (sf_id << 4);
                const uint64_t bd = encode_smem_desc(b0 + (kk >> 1) * b_bytes + (kk & 1) * 64, 16,
                                                     1024, SWZ_128B);
#pragma unroll
                for (int sub = 0; sub < MS; ++sub) {
                  const uint64_t ad =
                      encode_smem_desc(a0 + sub * a_bytes + kk * kMmaKBytes, 16, 1024, SWZ_128B);
                  mma_sp_bs<CG, KIND>(d_tmem + (uint32_t)(sub * BN), ad, bd,
                                e_tmem + (uint32_t)(MCOLS * sub + 2 * kk), id_k,
                                (sfa0 + 4u * sub) | (sf_id << 30), sfb | (sf_id << 30),
                                (kfirst | kk) != 0 ? 1u : 0u, on);
                }
              }
            }
          } else if constexpr (SPARSE) {
            // sub-tile `sub` of this slot: metadata columns e_tmem + MCOLS * sub
            const uint32_t e_tmem = meta_col0 + (uint32_t)(MCOLS * MS) * meta_slot;
#pragma unroll
            for (int sub = 0; sub < MS; ++sub)
#pragma unroll
              for (int hf = 0; hf < MCOLS / 4; ++hf)
                // 128 lanes x 16 bytes, no swizzle: 8-row core matrices 128 bytes apart
                tc_cp_128x128b<CG>(e_tmem + (uint32_t)(MCOLS * sub + 4 * hf),
                                   encode_smem_desc(sE + stage * side_bytes(VAR, MS, KIND) +
                                                        sub * MBYTES + 2048 * hf,
                                                    16, 128, SWZ_NONE),
                                   on);
            // Each MMA reads the compressed A's 32 bytes of K and 64 bytes of B per
            // row (dense K 16 for tf32, 32 for f16, 64 for the 8-bit kinds).  kind::f16
            // and kind::tf32 (whose pairs the metadata describes as groups of four
            // 16-bit halves): MMA kk reads metadata column e_tmem + kk; the instruction takes an even
            // column address and the descriptor's sparsity selector (bits 0-1)
            // picks the odd one.  8-bit kinds: MMA kk reads columns 2 kk, 2 kk + 1
            // (selector 0).  The loop stays rolled: a smaller loop body measured 1-2 %
            // faster per slot (clock stamps; cfg3 2787 against 2846 TFLOP/s).
            // (descriptors: the slot's first plus the start-address offset, as below)
            const uint64_t da0 = encode_smem_desc(a0, 16, 1024, SWZ_128B);
            const uint64_t db0 = encode_smem_desc(b0, 16, 1024, SWZ_128B);
#pragma unroll 1
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t bd = db0 + (uint64_t)(((kk >> 1) * b_bytes + (kk & 1) * 64) >> 4);
              const uint32_t e_col = MCOLS == 4 ? (uint32_t)(kk & ~1) : (uint32_t)(2 * kk);
              const uint32_t sel = MCOLS == 4 ? (uint32_t)(kk & 1) : 0u;
#pragma unroll
              for (int sub = 0; sub < MS; ++sub) {
                const uint64_t ad = da0 + (uint64_t)((sub * a_bytes + kk * kMmaKBytes) >> 4);
                const uint32_t e_addr = e_tmem + (uint32_t)(MCOLS * sub) + e_col;
                if constexpr (WS)
                  mma_ws_sp<KIND>(d_tmem, ad, bd, e_addr, idesc | sel,
                                  (kfirst | kk) != 0 ? 1u : 0u, on);
                else
                  mma_sp<CG, KIND>(d_tmem + (uint32_t)(sub * BN), ad, bd, e_addr, idesc | sel,
                                   (kfirst | kk) != 0 ? 1u : 0u, on);
              }
            }
          } else if constexpr (NVFP4) {
            const uint32_t dS = sE + stage * side_bytes(VAR, MS, KIND);
            const uint32_t dSfb = dS + MS * sfa_bytes(VAR);
            const uint32_t sf0 = meta_col0;  // the single scale-factor region (kSfRing = 1)
            // Kept rolled: the unrolled body (16 copies and 8 MMAs per NVFP4 slot) made
            // the MMA warp's loop 6 % slower per slot (clock stamps: 1104 against 1041
            // cycles; cfg4 5134 against 5304 TFLOP/s).
#pragma unroll 1
            for (int g = 0; g < SFG; ++g) {
              // group g: SFA of sub-tile `sub` at columns 4 * sub, the shared SFB at 4 * MS
              const uint32_t sfa0 = sf0 + (uint32_t)(sf_cols_per_slot(VAR, MS) / SFG) * g;
              const uint32_t sfb = sfa0 + 4u * MS;
              // 32 rows x 16 bytes, no swizzle: 8-row core matrices 128 bytes apart
              tc_cp_32x128b_warpx4<CG>(sfb, encode_smem_desc(dSfb + 1024 * g, 16, 128, SWZ_NONE),
                                       on);
              tc_cp_32x128b_warpx4<CG>(
                  sfb + 4u, encode_smem_desc(dSfb + 1024 * g + 512, 16, 128, SWZ_NONE), on);
#pragma unroll
              for (int sub = 0; sub < MS; ++sub)
                tc_cp_32x128b_warpx4<CG>(
                    sfa0 + 4u * sub,
                    encode_smem_desc(dS + sub * sfa_bytes(VAR) + 512 * g, 16, 128, SWZ_NONE), on);
#pragma unroll
              for (int m = 0; m < MPG; ++m) {
                const int kk = g * MPG + m;
                // the MMA's scales start at byte `sf_id` of each 32-bit column: carried
                // in the instruction descriptor (A bits 29-30, B bits 4-5) and in bits
                // 30-31 of the scale-factor TMEM addresses
                const uint32_t sf_id = (uint32_t)(m * SFG);
                const uint32_t id_k = idesc | (sf_id << 29) | (sf_id << 4);
                const uint64_t bd = encode_smem_desc(b0 + kk * kMmaKBytes, 16, 1024, SWZ_128B);
#pragma unroll
                for (int sub = 0; sub < MS; ++sub) {
                  const uint64_t ad =
                      encode_smem_desc(a0 + sub * a_bytes + kk * kMmaKBytes, 16, 1024, SWZ_128B);
                  mma_bs<CG, KIND>(d_tmem + (uint32_t)(sub * BN), ad, bd, id_k,
                                   (sfa0 + 4u * sub) | (sf_id << 30), sfb | (sf_id << 30),
                                   (kfirst | kk) != 0 ? 1u : 0u, on);
                }
              }
            }
          } else if constexpr (TS) {
            // A slice of each MMA (128 rows x 32 bytes) -> 8 TMEM columns, then the
            // MMA reads A from TMEM
            const uint32_t a_tm = meta_col0;
#pragma unroll
            for (int kk = 0; kk < kKBytes / kMmaKBytes; ++kk)
              tc_cp_128x256b<CG>(a_tm + 8u * kk,
                                 encode_smem_desc(a0 + kk * kMmaKBytes, 16, 1024, SWZ_128B), on);
#pragma unroll
            for (int kk = 0; kk < kKBytes / kMmaKBytes; ++kk) {
              const uint64_t bd = encode_smem_desc(b0 + kk * kMmaKBytes, 16, 1024, SWZ_128B);
              mma_ts<CG, KIND>(d_tmem, a_tm + 8u * kk, bd, idesc, (kfirst | kk) != 0 ? 1u : 0u, on);
            }
          } else {
            // dense: MS A sub-tiles share the slot's B (m_sub = 2 halves B's bytes
            // per MMA); KA K atoms per slot.  The descriptors of a slot differ only in
            // the start address field (address >> 4, 14 bits: shared memory stays below
            // 256 KB), so each is the slot's first descriptor plus a constant
            const uint64_t da0 = encode_smem_desc(a0, 16, 1024, SWZ_128B);
            const uint64_t db0 = encode_smem_desc(b0, 16, 1024, SWZ_128B);
#pragma unroll
            for (int t = 0; t < KA; ++t) {
#pragma unroll
              for (int kk = 0; kk < kKBytes / kMmaKBytes; ++kk) {
                const uint64_t bd = db0 + (uint64_t)((t * b_bytes + kk * kMmaKBytes) >> 4);
#pragma unroll
                for (int sub = 0; sub < MS; ++sub) {
                  const uint64_t ad =
                      da0 + (uint64_t)(((t * MS + sub) * a_bytes + kk * kMmaKBytes) >> 4);
                  const uint32_t acc_in = (kfirst | (uint32_t)t | (uint32_t)kk) != 0 ? 1u : 0u;
                  if constexpr (WS)
                    mma_ws_ss<KIND>(d_tmem, ad, bd, idesc, acc_in, on);
                  else
                    mma_ss<CG, KIND>(d_tmem + (uint32_t)(sub * BN), ad, bd, idesc, acc_in, on);
                }
              }
            }
          }
          if (CG == 2) tc_commit_mc<CG>(bar_empty + 8 * stage, 0x3, on);
          else tc_commit<CG>(bar_empty + 8 * stage, on);
          if (SPARSE) meta_slot = (meta_slot + 1) & (kMetaRing - 1);
          if (++stage == stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (issuer) {  // progress trace, per unit
          trace_store(trace, TR_FULL_SEEN, n_full);
          trace_store(trace, TR_MMA_ISSUED, n_full);
        }
        if (!ok) break;
        ++n_tiles;
        if (CG == 2) tc_commit_mc<CG>(bar_tfull + 8 * acc, 0x3, on);
        else tc_commit<CG>(bar_tfull + 8 * acc, on);
        if (issuer) trace_store(trace, TR_TILES_MMA, n_tiles);
        if (++acc == ACC) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Drain: wait until every MMA the elected lane issued has completed.
      int no_abort = 0;
      tc_commit<CG>(bar_drain, on);
      const bool drained = mbar_wait(bar_drain, 0, &no_abort, nullptr, 0, args.wait_ns);
      if (!drained && issuer) trace_store(trace, TR_TIMEOUTS, 16);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    const float alpha = args.alpha;
    __nv_bfloat16* C = args.C;
    const int64_t ldc = args.ldc;
    const bool vec_ok = args.c_vec_ok;
    uint32_t n_tfull = 0, n_done = 0;
    // M_SUB = 2: warp w also takes column half (w - 2) / 4 of the tile, [0, split)
    // or [split, BN) with split = BN / 2 rounded up to 16
    constexpr int NCH = epi_chunks(MS, VAR);
    const int split = ((BN / 2 + 15) / 16) * 16;
    const int c_lo = warp >= 6 ? split : 0;
    const int c_hi = warp >= 6 ? BN : split;
    for (int u = cluster_id; u < n_units; u += num_clusters) {
      const Unit w = unit_of(u, args);
      int mt, nt;
      tile_coords(w.tile, args.num_m_tiles, args.num_n_tiles, args.group_m, mt, nt);
      // every lane waits; the decision is made warp-uniform so that the
      // .sync.aligned TMEM loads below always run converged
      const bool got = mbar_wait(bar_tfull + 8 * acc, acc_phase, abort_flag, err,
                                 ERRW_TIMEOUT_EPILOGUE, args.wait_ns);
      if (!__all_sync(0xffffffffu, got)) {
        if (warp == 2 && lane == 0) trace_store(trace, TR_TIMEOUTS, 8);
        break;
      }
      if (warp == 2 && lane == 0) trace_store(trace, TR_TFULL_SEEN, ++n_tfull);
      tc_fence_after();
      const int row0 = mt * kRowsPerTile + (int)rank * kRowsPerCta * MS + quarter * 32 + lane;
      if constexpr (MS == 1) {
        // Double-buffered accumulator: stream 32-column chunks TMEM -> registers
        // -> C; tile i+1's MMAs run in the other buffer meanwhile.
        // Split tail: split s > 0 writes its fp32 partial rows instead of C and
        // stamps its flag; split 0 waits for every stamp and adds the partials.
        const int S = args.tail_split;
        const int ew = warp - 2;  // epilogue warp: this CTA's rows [32 ew, 32 ew + 32)
        // A warp's 32 rows x BN partial, laid out [32-column chunk][float4 v][lane] so
        // that every warp-wide float4 access covers 512 contiguous bytes.
        auto part_row = [&](int sp) -> float* {
          return args.part +
                 ((size_t)((w.vt * (S - 1) + sp - 1) * CG + (int)rank) * 4 + ew) * (size_t)(32 * BN) +
                 (size_t)lane * 4;
        };
        auto flag_of = [&](int sp) -> uint32_t* {
          return args.flags + ((size_t)(w.vt * (S - 1) + sp - 1) * CG + rank) * 4 + ew;
        };
        bool add_parts = false;
        if (w.vt >= 0 && w.split == 0) {
          bool okp = true;
          if (lane == 0)
            for (int sp = 1; sp < S && okp; ++sp)
              okp = wait_stamp(flag_of(sp), args.epoch, abort_flag, err, args.wait_ns);
          add_parts = __shfl_sync(0xffffffffu, okp ? 1 : 0, 0) != 0;
          __threadfence();
        }
        const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + (uint32_t)c0, r);
          tmem_ld_wait();
          if constexpr (KIND == KIND_I8) {
            // s32 accumulator -> fp32 (round to nearest even) before alpha; the
            // planner never splits an i8 tile, so no partials mix the two
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__int2float_rn((int)r[j]));
          }
          if (w.split > 0) {
            // chunk c0 / 32: float4 v of lane l at (c0 / 32 * 8 + v) * 128 + 4 l floats
            float* dst = part_row(w.split) + (size_t)c0 * 32;
#pragma unroll
            for (int v = 0; v < 8; ++v)
              __stcg(reinterpret_cast<float4*>(dst + v * 128),
                     make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                 __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3])));
            continue;
          }
          if (add_parts) {
            for (int sp = 1; sp < S; ++sp) {
              const float* src = part_row(sp) + (size_t)c0 * 32;
#pragma unroll
              for (int v = 0; v < 8; ++v) {
                const float4 q = __ldcg(reinterpret_cast<const float4*>(src + v * 128));
                r[4 * v] = __float_as_uint(__uint_as_float(r[4 * v]) + q.x);
                r[4 * v + 1] = __float_as_uint(__uint_as_float(r[4 * v + 1]) + q.y);
                r[4 * v + 2] = __float_as_uint(__uint_as_float(r[4 * v + 2]) + q.z);
                r[4 * v + 3] = __float_as_uint(__uint_as_float(r[4 * v + 3]) + q.w);
              }
            }
          }
          const int col = nt * BN + c0;
          if (row0 < args.M) {
            __nv_bfloat16* dst = C + (int64_t)row0 * ldc + col;
            if (vec_ok && col + 32 <= args.N) {
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                uint32_t w[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[v * 8 + 2 * j]) * alpha,
                                                           __uint_as_float(r[v * 8 + 2 * j + 1]) * alpha);
                  w[j] = *reinterpret_cast<uint32_t*>(&h);
                }
                *reinterpret_cast<uint4*>(dst + v * 8) = make_uint4(w[0], w[1], w[2], w[3]);
              }
            } else {
              for (int j = 0; j < 32; ++j)
                if (col + j < args.N) dst[j] = __float2bfloat16_rn(__uint_as_float(r[j]) * alpha);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (CG == 2) mbar_arrive_cluster(mapa_shared(bar_tempty + 8 * acc, 0));
          else mbar_arrive(bar_tempty + 8 * acc);
          if (w.split > 0) {
            // the warp's partial rows are written (ordered by the warp barrier):
            // publish them at GPU scope
            __threadfence();
            asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(flag_of(w.split)),
                         "r"(args.epoch)
                         : "memory");
          }
        }
      } else if constexpr (VAR == VAR_DENSE && KIND == KIND_F16) {
        // One accumulator buffer, dense 16-bit operands: this warp's part of both
        // sub-tiles streams TMEM -> registers -> C, kEpiGroup 16-column loads per
        // tcgen05.wait::ld (4 round trips per warp instead of 16; the stores need no
        // registers kept across loads), and TMEM goes back to the MMA issuer as soon
        // as the tile's last loads have landed.  The MMA issuer waits for that at
        // every tile start.  Measured at bf16 8192^3 against the read-all-then-store
        // form below: +3.6 % in bursts; for fp8 (tiles half as long, so C is stored
        // twice as fast) the stores issued before the release held it back (-2 %), so
        // the other kinds keep the form below.
        constexpr int kEpiGroup = 4;
#pragma unroll
        for (int sub = 0; sub < MS; ++sub) {
          const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) +
                                 (uint32_t)((acc * MS + sub) * BN);
          const int row = row0 + sub * kRowsPerCta;
#pragma unroll
          for (int j0 = 0; j0 < NCH; j0 += kEpiGroup) {
            uint32_t r[kEpiGroup][16];
#pragma unroll
            for (int g = 0; g < kEpiGroup; ++g) {
              const int c0 = c_lo + 16 * (j0 + g);
              if (j0 + g < NCH && c0 < c_hi)  // warp-uniform
                tmem_ld_32x32b_x16(t_row + (uint32_t)c0, r[g]);
            }
            tmem_ld_wait();
            if (sub == MS - 1 && j0 + kEpiGroup >= NCH) {
              // the tile's last TMEM loads are in registers: release the accumulator
              tc_fence_before();
              __syncwarp();
              if (lane == 0) {
                if (CG == 2) mbar_arrive_cluster(mapa_shared(bar_tempty + 8 * acc, 0));
                else mbar_arrive(bar_tempty + 8 * acc);
              }
            }
#pragma unroll
            for (int g = 0; g < kEpiGroup; ++g) {
              const int c0 = c_lo + 16 * (j0 + g);
              if (j0 + g >= NCH || c0 >= c_hi || row >= args.M) continue;
              uint32_t w[8];
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[g][2 * q]) * alpha,
                                                         __uint_as_float(r[g][2 * q + 1]) * alpha);
                w[q] = *reinterpret_cast<uint32_t*>(&h);
              }
              const int col = nt * BN + c0;
              __nv_bfloat16* dst = C + (int64_t)row * ldc + col;
              if (vec_ok && col + 16 <= args.N) {
#pragma unroll
                for (int v = 0; v < 2; ++v)
                  *reinterpret_cast<uint4*>(dst + v * 8) =
                      make_uint4(w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
              } else {
#pragma unroll
                for (int e = 0; e < 16; ++e)
                  if (col + e < args.N)
                    dst[e] = __ushort_as_bfloat16((unsigned short)(w[e >> 1] >> (16 * (e & 1))));
              }
            }
          }
        }
      } else {
        // One accumulator buffer: read this warp's part of both sub-tiles into
        // registers as packed bf16, release TMEM, then store, so that the stores
        // of tile i run under the MMAs of tile i+1.
        uint32_t pk[MS][NCH][8];  // this lane's row, 16 columns per chunk, bf16 pairs
#pragma unroll
        for (int sub = 0; sub < MS; ++sub) {
          const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) +
                                 (uint32_t)((acc * MS + sub) * BN);
#pragma unroll
          for (int j = 0; j < NCH; ++j) {
            const int c0 = c_lo + 16 * j;
            if (c0 < c_hi) {  // warp-uniform
              uint32_t r[16];
              tmem_ld_32x32b_x16(t_row + (uint32_t)c0, r);
              tmem_ld_wait();
              if constexpr (KIND == KIND_I8) {  // s32 accumulator -> fp32 before alpha
#pragma unroll
                for (int q = 0; q < 16; ++q) r[q] = __float_as_uint(__int2float_rn((int)r[q]));
              }
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[2 * q]) * alpha,
                                                         __uint_as_float(r[2 * q + 1]) * alpha);
                pk[sub][j][q] = *reinterpret_cast<uint32_t*>(&h);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (CG == 2) mbar_arrive_cluster(mapa_shared(bar_tempty + 8 * acc, 0));
          else mbar_arrive(bar_tempty + 8 * acc);
        }
#pragma unroll
        for (int sub = 0; sub < MS; ++sub) {
          const int row = row0 + sub * kRowsPerCta;
          if (row >= args.M) continue;
#pragma unroll
          for (int j = 0; j < NCH; ++j) {
            const int c0 = c_lo + 16 * j;
            if (c0 >= c_hi) continue;
            const int col = nt * BN + c0;
            __nv_bfloat16* dst = C + (int64_t)row * ldc + col;
            if (vec_ok && col + 16 <= args.N) {
#pragma unroll
              for (int v = 0; v < 2; ++v)
                *reinterpret_cast<uint4*>(dst + v * 8) =
                    make_uint4(pk[sub][j][4 * v], pk[sub][j][4 * v + 1], pk[sub][j][4 * v + 2],
                               pk[sub][j][4 * v + 3]);
            } else {
#pragma unroll
              for (int e = 0; e < 16; ++e)
                if (col + e < args.N)
                  dst[e] = __ushort_as_bfloat16((unsigned short)(pk[sub][j][e >> 1] >> (16 * (e & 1))));
            }
          }
        }
      }
      if (warp == 2 && lane == 0) trace_store(trace, TR_TILES_EPI, ++n_done);
      if (++acc == ACC) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  // ------------------------------------------------------------ teardown
  __syncwarp();
  if (threadIdx.x == 0) trace_store(trace, TR_STAGE, 5);
  tc_fence_before();
  __syncthreads();
  if (CG == 2) cluster_sync();
  tc_fence_after();
  if (threadIdx.x == 0) trace_store(trace, TR_STAGE, 6);
  if (warp == 1) {
    tmem_dealloc<CG>(tmem_base, tmem_cols);
    if (lane == 0) trace_store(trace, TR_STAGE, 7);
  }
}

// ---------------------------------------------------------------- launchers
size_t gemm_smem_bytes(int stages, int b_rows, int var, int m_sub, int k_atoms, int kind) {
  return (size_t)carve(stages, b_rows, var, m_sub, k_atoms, kind).total + 1024;  // + alignment slack
}

int gemm_kernel_threads(int m_sub) { return kernel_threads(m_sub); }

int gemm_tmem_columns(int tile_n, int var, bool ts, int m_sub, int kind) {
  return (int)tmem_columns(tile_n, var, ts, m_sub, kind);
}

int gemm_default_m_sub(int var, int64_t M, int64_t N, int64_t K, int cg, int tile_n,
                       int clusters) {
  if (K < 2048) return 1;
  const int64_t n_tiles = (N + tile_n - 1) / tile_n;
  const int64_t tiles2 = ((M + 256 * cg - 1) / (256 * cg)) * n_tiles;
  if (var == VAR_DENSE) {
    // dense: two sub-tiles only on 256-column pair tiles (512 x 256, the 2 x 256
    // accumulator columns fill TMEM) with K >= 8192 (the single accumulator's drain,
    // about 3k cycles per tile, is then near 5 % of a tile), and only where the waves
    // of 512-row tiles take no more time than those of 256-row ones (each is twice as
    // long) and number at least 4 (a short grid keeps the split tail).  Measured at
    // 8192^3 against 256 x 256 pair tiles, interleaved: bf16 +5.4 % in short bursts
    // and +6 % power-capped, e4m3 +1.9 % and +1.5 %; the 512-row tile moves a quarter
    // fewer L2 -> shared-memory bytes per MMA and runs at a higher clock under the cap.
    if (cg != 2 || tile_n != 256 || K < 8192) return 1;
    const int64_t tiles1 = ((M + 128 * cg - 1) / (128 * cg)) * n_tiles;
    const int64_t w1 = (tiles1 + clusters - 1) / clusters, w2 = (tiles2 + clusters - 1) / clusters;
    return (2 * w2 <= w1 && w2 >= 4) ? 2 : 1;
  }
  return tiles2 >= clusters ? 2 : 1;
}

template <int CG>
static cudaLaunchConfig_t make_cfg(int grid, int threads, size_t smem, cudaStream_t stream,
                                   cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CG;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// Largest dynamic shared memory already allowed for a kernel instance, per device
// (devices 0..7; others set the attribute on every launch): the attribute is raised
// only when a launch needs more, not set again on every call.
constexpr int kSmemAttrDevices = 8;

template <int KIND, int CG, int VAR, bool TS, int MS, int KA = 1, bool WS = false>
static cudaError_t launch_one(const GemmMaps& m, const GemmArgs& a, int grid, size_t smem,
                              cudaStream_t stream, int* max_clusters) {
  auto* fn = gemm_tn_kernel<KIND, CG, VAR, TS, MS, KA, WS>;
  static std::atomic<int> smem_set[kSmemAttrDevices];
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const bool cached = dev >= 0 && dev < kSmemAttrDevices;
  if (!cached || smem_set[dev].load(std::memory_order_relaxed) < (int)smem) {
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    if (cached) {  // keep the largest value set
      int cur = smem_set[dev].load(std::memory_order_relaxed);
      while (cur < (int)smem && !smem_set[dev].compare_exchange_weak(cur, (int)smem)) {
      }
    }
  }
  cudaLaunchAttribute attr[1];
  if (max_clusters) {  // occupancy query only
    cudaLaunchConfig_t cfg = make_cfg<CG>(2 * CG, kernel_threads(MS), smem, nullptr, attr);
    return cudaOccupancyMaxActiveClusters(max_clusters, fn, &cfg);
  }
  cudaLaunchConfig_t cfg = make_cfg<CG>(grid, kernel_threads(MS), smem, stream, attr);
  e = cudaLaunchKernelEx(&cfg, fn, m.a, m.b, m.e, m.f, m.g, a);
  if (e == cudaErrorInvalidValue && cached) {
    // the attribute no longer holds (the device was reset): set it again and retry
    (void)cudaGetLastError();
    smem_set[dev].store(0, std::memory_order_relaxed);
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    smem_set[dev].store((int)smem, std::memory_order_relaxed);
    e = cudaLaunchKernelEx(&cfg, fn, m.a, m.b, m.e, m.f, m.g, a);
  }
  return e;
}

template <int KIND, int VAR, bool TS, int MS = 1, int KA = 1>
static cudaError_t launch_cg(int cg, const GemmMaps& m, const GemmArgs& a, int grid, size_t smem,
                             cudaStream_t s, int* mc) {
  return cg == 2 ? launch_one<KIND, 2, VAR, TS, MS, KA>(m, a, grid, smem, s, mc)
                 : launch_one<KIND, 1, VAR, TS, MS, KA>(m, a, grid, smem, s, mc);
}

// Instances built: dense f16 / f8f6f4 (SS and TS), dense tf32 / i8 (SS), sparse
// f16 and the block-scaled kinds (one or two A sub-tiles each); cta_group 1 and 2
// each.  The f8f6f4 instance serves every element type of that kind (e4m3, e5m2,
// e2m3, e3m2, e2m1): the type lives in the runtime instruction descriptor.  `mc` non-null turns a call into
// the occupancy query.
static cudaError_t dispatch(int kind, int cg, int var, bool ts, int m_sub, int k_atoms, bool ws,
                            const GemmMaps& m, const GemmArgs& a, int grid, size_t smem,
                            cudaStream_t s, int* mc) {
  if (ws) {  // tcgen05.mma.ws{.sp}: cta_group::1, SS, one sub-tile, one K atom
    const bool sp = var == VAR_SPARSE;
    switch (kind) {
      case KIND_TF32:
        return sp ? launch_one<KIND_TF32, 1, VAR_SPARSE, false, 1, 1, true>(m, a, grid, smem, s, mc)
                  : launch_one<KIND_TF32, 1, VAR_DENSE, false, 1, 1, true>(m, a, grid, smem, s, mc);
      case KIND_F16:
        return sp ? launch_one<KIND_F16, 1, VAR_SPARSE, false, 1, 1, true>(m, a, grid, smem, s, mc)
                  : launch_one<KIND_F16, 1, VAR_DENSE, false, 1, 1, true>(m, a, grid, smem, s, mc);
      case KIND_F8F6F4:
        return sp ? launch_one<KIND_F8F6F4, 1, VAR_SPARSE, false, 1, 1, true>(m, a, grid, smem, s, mc)
                  : launch_one<KIND_F8F6F4, 1, VAR_DENSE, false, 1, 1, true>(m, a, grid, smem, s, mc);
      default:
        return sp ? launch_one<KIND_I8, 1, VAR_SPARSE, false, 1, 1, true>(m, a, grid, smem, s, mc)
                  : launch_one<KIND_I8, 1, VAR_DENSE, false, 1, 1, true>(m, a, grid, smem, s, mc);
    }
  }
  if (k_atoms == 2) {  // dense SS, one sub-tile, two K atoms per slot
    switch (kind) {
      case KIND_F16: return launch_cg<KIND_F16, VAR_DENSE, false, 1, 2>(cg, m, a, grid, smem, s, mc);
      case KIND_F8F6F4: return launch_cg<KIND_F8F6F4, VAR_DENSE, false, 1, 2>(cg, m, a, grid, smem, s, mc);
      case KIND_TF32: return launch_cg<KIND_TF32, VAR_DENSE, false, 1, 2>(cg, m, a, grid, smem, s, mc);
      default: return launch_cg<KIND_I8, VAR_DENSE, false, 1, 2>(cg, m, a, grid, smem, s, mc);
    }
  }
  if (var == VAR_SPARSE) {  // structured-sparse A: kind::f16, f8f6f4, i8 (2:4), tf32 (1:2)
    if (kind == KIND_TF32)
      return m_sub == 2 ? launch_cg<KIND_TF32, VAR_SPARSE, false, 2>(cg, m, a, grid, smem, s, mc)
                        : launch_cg<KIND_TF32, VAR_SPARSE, false, 1>(cg, m, a, grid, smem, s, mc);
    if (kind == KIND_F8F6F4)
      return m_sub == 2 ? launch_cg<KIND_F8F6F4, VAR_SPARSE, false, 2>(cg, m, a, grid, smem, s, mc)
                        : launch_cg<KIND_F8F6F4, VAR_SPARSE, false, 1>(cg, m, a, grid, smem, s, mc);
    if (kind == KIND_I8)
      return m_sub == 2 ? launch_cg<KIND_I8, VAR_SPARSE, false, 2>(cg, m, a, grid, smem, s, mc)
                        : launch_cg<KIND_I8, VAR_SPARSE, false, 1>(cg, m, a, grid, smem, s, mc);
    return m_sub == 2 ? launch_cg<KIND_F16, VAR_SPARSE, false, 2>(cg, m, a, grid, smem, s, mc)
                      : launch_cg<KIND_F16, VAR_SPARSE, false, 1>(cg, m, a, grid, smem, s, mc);
  }
  if (var == GEMM_NVFP4_SP)  // 4:8-sparse A in pairs on kind::mxf4nvf4 (block16)
    return m_sub == 2
               ? launch_cg<KIND_MXF4NVF4, GEMM_NVFP4_SP, false, 2>(cg, m, a, grid, smem, s, mc)
               : launch_cg<KIND_MXF4NVF4, GEMM_NVFP4_SP, false, 1>(cg, m, a, grid, smem, s, mc);
  if (var == GEMM_MXF4_SP)  // 4:8-sparse A in pairs on kind::mxf4
    return m_sub == 2
               ? launch_cg<KIND_MXF4, GEMM_MXF4_SP, false, 2>(cg, m, a, grid, smem, s, mc)
               : launch_cg<KIND_MXF4, GEMM_MXF4_SP, false, 1>(cg, m, a, grid, smem, s, mc);
  if (var == GEMM_MXF8_SP)  // 2:4-sparse A on kind::mxf8f6f4
    return m_sub == 2
               ? launch_cg<KIND_MXF8F6F4, GEMM_MXF8_SP, false, 2>(cg, m, a, grid, smem, s, mc)
               : launch_cg<KIND_MXF8F6F4, GEMM_MXF8_SP, false, 1>(cg, m, a, grid, smem, s, mc);
  if (var == VAR_NVFP4)
    return m_sub == 2 ? launch_cg<KIND_MXF4NVF4, VAR_NVFP4, false, 2>(cg, m, a, grid, smem, s, mc)
                      : launch_cg<KIND_MXF4NVF4, VAR_NVFP4, false, 1>(cg, m, a, grid, smem, s, mc);
  if (var == GEMM_MXF8)
    return m_sub == 2 ? launch_cg<KIND_MXF8F6F4, GEMM_MXF8, false, 2>(cg, m, a, grid, smem, s, mc)
                      : launch_cg<KIND_MXF8F6F4, GEMM_MXF8, false, 1>(cg, m, a, grid, smem, s, mc);
  if (var == GEMM_MXF4)
    return m_sub == 2 ? launch_cg<KIND_MXF4, GEMM_MXF4, false, 2>(cg, m, a, grid, smem, s, mc)
                      : launch_cg<KIND_MXF4, GEMM_MXF4, false, 1>(cg, m, a, grid, smem, s, mc);
  if (m_sub == 2) {  // dense, two A sub-tiles per CTA (f16 and f8f6f4 kinds)
    if (kind == KIND_F16) return launch_cg<KIND_F16, VAR_DENSE, false, 2>(cg, m, a, grid, smem, s, mc);
    return launch_cg<KIND_F8F6F4, VAR_DENSE, false, 2>(cg, m, a, grid, smem, s, mc);
  }
  if (kind == KIND_F16)
    return ts ? launch_cg<KIND_F16, VAR_DENSE, true>(cg, m, a, grid, smem, s, mc)
              : launch_cg<KIND_F16, VAR_DENSE, false>(cg, m, a, grid, smem, s, mc);
  if (kind == KIND_TF32) return launch_cg<KIND_TF32, VAR_DENSE, false>(cg, m, a, grid, smem, s, mc);
  if (kind == KIND_I8) return launch_cg<KIND_I8, VAR_DENSE, false>(cg, m, a, grid, smem, s, mc);
  return ts ? launch_cg<KIND_F8F6F4, VAR_DENSE, true>(cg, m, a, grid, smem, s, mc)
            : launch_cg<KIND_F8F6F4, VAR_DENSE, false>(cg, m, a, grid, smem, s, mc);
}

cudaError_t gemm_max_active_clusters(int kind, int cg, int var, bool ts, int m_sub, int k_atoms,
                                     bool ws, int smem, int* out) {
  GemmMaps m;
  GemmArgs a;
  return dispatch(kind, cg, var, ts, m_sub, k_atoms, ws, m, a, 0, (size_t)smem, nullptr, out);
}

cudaError_t gemm_launch(int kind, int cg, int var, bool ts, int m_sub, int k_atoms, bool ws,
                        const GemmMaps& m, const GemmArgs& a, int grid, size_t smem,
                        cudaStream_t s) {
  return dispatch(kind, cg, var, ts, m_sub, k_atoms, ws, m, a, grid, smem, s, nullptr);
}

}  // namespace b2g
