// Warp-specialized, persistent tensor-core GEMM (tcgen05 kind::i8) for the fused quantize + GEMM path with many
// activation columns (M >= 8: prefill, batched or speculative decode).
//
// Same results as gemm_tc.cu and the GEMVs: every int32 block dot is exact, and Y adds the per-block f32 products in
// the reference's multiply order (Q4_0 / Q8_0: f32(s) * dw * dx; TQ2_0: dx * dw * f32(s); kernels.py:93, 141), blocks
// in ascending order -- so Y is bit-identical to the other schedules. What changes is who does what:
//   * a prep kernel quantizes the f32 activations with the math of b2q_quant_q8_0 / b2q_quant_q8_K straight into the
//     MMA operand layout (per column tile of NT columns and 32-value unit: one NT x 32-byte K-major tile of 8 x 16-byte
//     core matrices), and writes per column and weight block the scale dx;
//   * warp 8 (producer) streams per stage -- 128 packed weight bytes of each of the tile's 128 rows -- the rows'
//     weights (one 2-D TMA tensor copy of a 128-row x 128-byte box, 128-byte swizzled so that the unpacking reads are
//     free of bank conflicts; rows past N read as zeros) and the stage's activation tiles (one bulk copy) into a ring
//     of P stages, and its column scales (one bulk copy) into a deeper ring of their own: the epilogue reads them up
//     to two stages behind the MMAs, and a weight stage must not wait for it to be refilled;
//   * warps 4-7 (thread r = tile row r) unpack each 32-value unit of their row into the MMA's A tile (a ring of RA
//     tiles) as the signed weight values (Q4_0 nibble - 8, TQ2_0 crumb - 1), so the tensor cores' int32 dots are the
//     exact block dots with no offset term;
//   * one thread of warp 9 issues each unit's MMA (M = 128, N = NT, K = 32) into its block's accumulator (a ring of
//     RT accumulators in tensor memory) and commits completions to the mbarriers the other roles wait on;
//   * warps 0-3 (thread t = tile row t = tensor-memory lane t) run each weight block's epilogue: its NT exact int32
//     dots from tensor memory, converted exactly (2^23 + 2^22 + s as f32 bits by one integer add, valid for
//     |s| < 2^22), scaled and summed into NT f32 registers in block order; each row's block scales come through a
//     per-thread cp.async ring.
// Unpacking and epilogue run in separate warps so that their latency chains overlap (measured: with one set of warps
// doing both, each 32-value unit cost the sum of both chains and the MMA warp sat idle most of the time).
// The CTAs are persistent: CTA i takes the (row tile, column tile) pairs i, i + gridDim.x, ...; the stage ring and
// the unit / block counters run on across tile boundaries. Roles synchronize only through mbarriers (no CTA barrier in
// the loop). Every wait is bounded: a timeout sets the device error word and ends all roles, which then wait (bounded)
// for their copies and MMAs in flight, and the tensor memory is freed.
#include <cuda.h>

#include <mutex>

#include "tc_device.cuh"

namespace b2q {

struct WsParams {
  CUtensorMap wmap;   // the weights' quant plane as a 2-D byte tensor [N][row bytes], 128 x 128-byte boxes, 128B swizzle
  const uint8_t* wq;
  int64_t ldwq;
  const int16_t* ws;
  int64_t ldws;
  const int8_t* xt;   // activation tiles [nct][K/32][NT*32]
  const float* dk;    // [nct][nblk][NT]: the column scales dx
  const int* fk;      // TQ2_0: [nct][nblk][NT]: each accumulator's start value, 2^23 + 2^22 - sum(x) of the block
  float* y;
  int64_t ldy;
  int64_t row0;
  int64_t N;
  int64_t K;
  int M;
  int nct;     // column tiles
  int ks;      // K splits (split-K for layers whose row tiles alone do not fill the GPU)
  int ntiles;  // row tiles x column tiles x K splits
  float* part; // ks > 1: the splits' partial sums [ks][M][N]; a combine kernel adds them in split order into Y
};

// Pipeline shape per weight format and column tile. A stage is 128 packed weight bytes of each row: 8 Q4_0 blocks,
// 2 TQ2_0 blocks or 4 Q8_0 blocks (SU 32-value units). Roles hand work over in groups of GU units (one barrier phase,
// one fence and one commit per group, not per unit). P is chosen so that two CTAs fit on an SM where the registers
// allow it (NT <= 32).
template <int FMT, int NT>
struct WsCfg {
  static constexpr int UPB = FMT == 1 ? 8 : 1;                    // units per weight block
  static constexpr int WU = FMT == 0 ? 16 : FMT == 1 ? 8 : 32;   // packed weight bytes per unit and row
  static constexpr int RB = 128;                                  // packed weight bytes per row and stage
  static constexpr int SU = RB / WU;                              // units per stage
  static constexpr int SB = SU / UPB;                             // weight blocks per stage
  static constexpr int RAW = 128 * RB;                            // the weight box (128B-swizzled rows)
  static constexpr int BT = NT * 32;                              // one unit's activation tile
  static constexpr int BST = SU * BT;
  static constexpr int DKB = NT * 4;                              // column scales of one block
  static constexpr int DKS = SB * DKB;
  // TQ2_0: the crumbs' offset (-1) enters through the accumulators' start value (2^23 + 2^22 - sum(x) per column and
  // block) instead of offset MMAs; each column-scale ring entry also carries the start values of the blocks that next
  // use the stage's accumulators (RT blocks later)
  static constexpr bool FILL = FMT == 1;
  static constexpr int DKR = DKS + (FILL ? DKS : 0);  // column-scale ring entry
  static constexpr int OT = FMT == 0 ? 1 : 0;          // the offset tile (Q4_0)
  static constexpr int STAGE = (RAW + BST + 1023) / 1024 * 1024;  // swizzled boxes start on 1024 bytes
  static constexpr int P = FMT == 0 ? (NT == 16 ? 3 : NT == 32 ? 2 : NT == 64 ? 4 : 3)
                                    : FMT == 1 ? (NT == 16 || NT == 64 ? 3 : 2) : (NT <= 32 ? 3 : 4);
  static constexpr int GU = NT == 128 && UPB == 1 ? 2 : 4;         // units per hand-over group
  static constexpr int RAG = 2;                                   // A-tile groups in flight
  static constexpr int RA = RAG * GU;                             // A tiles
  static constexpr int ATILE = 128 * 32;
  // blocks per accumulator group (one epilogue hand-over each): a whole stage for Q4_0 and TQ2_0 at 16 columns
  // (measured faster than groups of 4 blocks, or of one TQ2_0 block), else GU
  static constexpr int AG = (FMT != 2 && NT == 16) ? SB : UPB == 1 ? GU : 1;
  static constexpr int RTG = NT == 16 ? 16 / AG : 2;  // accumulator groups in flight (16 x NT tensor-memory columns)
  static constexpr int RT = RTG * AG;                             // accumulators (blocks) in tensor memory
  static constexpr int CW = NT == 64 ? 32 : 16;                   // columns per tensor-memory load (registers)
  static constexpr int SBB = SB * 2;                              // scale bytes per row and stage (16, 4 or 8)
  static constexpr int PS = 3, LA = 2;                            // scale ring depth, prefetch distance (stages)
  // column-scale ring (stages): the epilogue trails the MMAs by up to RTG accumulator groups, so the column scales
  // live in their own, deeper ring and a weight stage is refilled as soon as its unpacking and MMAs are done
  static constexpr int PD = P + (RTG * AG + SB - 1) / SB + 1;
  static constexpr int TCOLS = RT * NT <= 32 ? 32 : RT * NT <= 64 ? 64 : RT * NT <= 128 ? 128 : RT * NT <= 256 ? 256
                                                                                                           : 512;
  // + 1024: the kernel aligns its base to 1024 bytes (the swizzle pattern follows the shared-memory address bits)
  static constexpr size_t SMEM =
      (size_t)P * STAGE + (size_t)(RA + OT) * ATILE + (size_t)PS * 128 * SBB + (size_t)PD * DKR + 1024;
  // registers are allocated per SM sub-partition (16K each) and a CTA's 10 warps land on them 3, 3, 2, 2: two CTAs
  // put 6 warps on one sub-partition, so two CTAs per SM need at most 85 registers a thread; one CTA at most 170
  static constexpr int MAXREG = NT <= 32 ? 80 : 168;
  static_assert(PS >= LA + 1, "scale ring: the slot refilled at a stage's start is no longer read");
  static_assert(SU % GU == 0 && SB % AG == 0 && (UPB == 1 || UPB % GU == 0), "groups never straddle stages");
  static_assert(RT * NT <= 512 && NT % 16 == 0 && CW % 16 == 0, "tensor memory");
  static_assert(FMT != 0 || (AG * NT <= 256 && RT % AG == 0 && SU % AG == 0), "Q4_0: one offset MMA per group");
  static_assert(!FILL || (RT % SB == 0 && NT % 16 == 0), "start values travel a whole number of stages ahead");
  static_assert(!FILL || (RT * NT * 4 <= PS * 128 * SBB && RT * NT <= 256), "first start values staged in the scale ring");
};

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// 2-D TMA tensor copy of the box at (x bytes, y rows) into this CTA's shared memory (the weights: this GPU's own
// memory), completion counted in bytes on `bar`
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar,
                                            uint64_t pol, bool hint) {
  const uint64_t m = reinterpret_cast<uint64_t>(map);
  if (hint)
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
        "%3}], [%4], %5;" ::"r"(dst),
        "l"(m), "r"(x), "r"(y), "r"(bar), "l"(pol)
        : "memory");
  else
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(dst),
        "l"(m), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void bulk_g2s_plain(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// One 32-value unit of row r -> its row of an A tile in value order: Q4_0 nibbles and TQ2_0 crumbs as unsigned bytes
// (their offsets -8 / -1 enter through a second MMA on the offset tile), Q8_0 weights as stored.
// raw: the row's 128 bytes of the stage, whose 16-byte chunk c sits at chunk c ^ (r % 8) (TMA 128B swizzle).
template <int FMT>
__device__ __forceinline__ void unpack_unit(uint32_t raw, int sw, int u, uint8_t* at, int r, const uint4 (&tq)[2]) {
  uint4 lo, hi;
  if (FMT == 0) {
    const uint4 w = lds_v4(raw + (uint32_t)((u ^ sw) << 4));
    constexpr uint32_t m = 0x0F0F0F0Fu;
    lo = make_uint4(w.x & m, w.y & m, w.z & m, w.w & m);
    hi = make_uint4((w.x >> 4) & m, (w.y >> 4) & m, (w.z >> 4) & m, (w.w >> 4) & m);
  } else if (FMT == 2) {
    lo = lds_v4(raw + (uint32_t)(((2 * u) ^ sw) << 4));
    hi = lds_v4(raw + (uint32_t)(((2 * u + 1) ^ sw) << 4));
  } else {  // TQ2_0 k-step s = u % 8 of a block: values 32s..32s+31 = field s % 4 of the (preloaded) 32 bytes tq
    const int sh = 2 * (u & 3);
    auto crumb = [sh](uint32_t x) { return (x >> sh) & 0x03030303u; };
    lo = make_uint4(crumb(tq[0].x), crumb(tq[0].y), crumb(tq[0].z), crumb(tq[0].w));
    hi = make_uint4(crumb(tq[1].x), crumb(tq[1].y), crumb(tq[1].z), crumb(tq[1].w));
  }
  *reinterpret_cast<uint4*>(at + tc::core_off(r, 0)) = lo;
  *reinterpret_cast<uint4*>(at + tc::core_off(r, 16)) = hi;
}

template <int FMT, int NT>
__global__ void __launch_bounds__(320) __maxnreg__((WsCfg<FMT, NT>::MAXREG))
    gemm_tc_ws_kernel(const __grid_constant__ WsParams p) {
  using C = WsCfg<FMT, NT>;
  constexpr int P = C::P, SU = C::SU, SB = C::SB, RA = C::RA, RT = C::RT, UPB = C::UPB, PS = C::PS, LA = C::LA;
  constexpr int GU = C::GU, RAG = C::RAG, AG = C::AG, RTG = C::RTG;
  extern __shared__ __align__(1024) uint8_t ws_smem[];
  __shared__ __align__(8) uint64_t bar_full[P], bar_empty[P], bar_afull[RAG], bar_aempty[RAG], bar_accf[RTG],
      bar_acce[RTG], bar_dkf[C::PD], bar_dke[C::PD], bar_tinit;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;

  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const uint32_t sbase = (smem_addr(ws_smem) + 1023u) & ~1023u;
  const uint32_t a_base = sbase + P * C::STAGE;
  const uint32_t off_tile = a_base + RA * C::ATILE;  // the weight offset (-8 or -1) in every byte
  const uint32_t sc_base = off_tile + C::OT * C::ATILE;
  const uint32_t dk_base = sc_base + PS * 128 * C::SBB;  // column-scale ring, PD entries of DKR bytes
  const int nunits = (int)(p.K / 32);
  const int nblk = (int)(p.K / Fmt<FMT>::kBlock);
  const int S = nunits / SU / p.ks;  // stages per tile (its K split)
  const int nbt = nblk / p.ks;       // weight blocks per tile
  const int my_tiles = (int)blockIdx.x < p.ntiles ? (p.ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int total_stages = my_tiles * S;
  volatile int* abort_flag = &s_abort;
  // the abort flag as lane 0 of the warp sees it, so that every lane takes the same branch (full-warp syncs follow)
  auto aborted = [&]() { return __shfl_sync(0xffffffffu, *abort_flag, 0) != 0; };

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                 "n"(C::TCOLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (t == 0) {
    for (int i = 0; i < P; ++i) {
      mbar_init(smem_addr(&bar_full[i]), 1);
      mbar_init(smem_addr(&bar_empty[i]), 4 + 1);  // unpack warps, the MMA commit
    }
    for (int i = 0; i < C::PD; ++i) {
      mbar_init(smem_addr(&bar_dkf[i]), 1);
      mbar_init(smem_addr(&bar_dke[i]), 4);  // epilogue warps
    }
    mbar_init(smem_addr(&bar_tinit), 4);  // epilogue warps: the accumulators hold the conversion constant
    for (int i = 0; i < RAG; ++i) {
      mbar_init(smem_addr(&bar_afull[i]), 4);
      mbar_init(smem_addr(&bar_aempty[i]), 1);
    }
    for (int i = 0; i < RTG; ++i) {
      mbar_init(smem_addr(&bar_accf[i]), 1);
      mbar_init(smem_addr(&bar_acce[i]), 4);
    }
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = s_tmem;

  // (row tile, column tile, stage along K) of this CTA's global stage G; a tile is (row tile, column tile, K split)
  auto stage_tile = [&](int G, int& rt, int& ct, int& s) {
    const int k = G / S;
    const int tile = (int)blockIdx.x + k * (int)gridDim.x;
    const int rc = tile / p.ks, kq = tile - rc * p.ks;
    s = kq * S + (G - k * S);
    rt = rc / p.nct;
    ct = rc - rt * p.nct;
  };

  int issued = 0;    // producer: stages whose copies were issued
  int g_issued = 0;  // MMA thread: unit groups issued
  if (warp == 8) {
    // ---------------- producer ----------------
    const bool stream_once = p.nct == 1;  // several column tiles re-read the weights from L2: no evict-first hint
    const uint64_t pol = evict_first_policy();
    auto issue_weights = [&](int G) {
      if (lane == 0) {
        int rt, ct, s;
        stage_tile(G, rt, ct, s);
        const uint32_t bar = smem_addr(&bar_full[G % P]);
        // the whole box counts, rows past N included (filled with zeros)
        mbar_expect_tx(bar, (uint32_t)(C::RAW + C::BST));
        tma_load_2d(sbase + (uint32_t)((G % P) * C::STAGE), &p.wmap, s * C::RB, rt * 128, bar, pol, stream_once);
      }
    };
    auto issue_acts = [&](int G) {
      if (lane == 0) {
        int rt, ct, s;
        stage_tile(G, rt, ct, s);
        const uint32_t bar = smem_addr(&bar_full[G % P]);
        const uint32_t st = sbase + (uint32_t)((G % P) * C::STAGE);
        bulk_g2s_plain(st + C::RAW, p.xt + ((int64_t)ct * nunits + (int64_t)s * SU) * C::BT, C::BST, bar);
        const uint32_t dbar = smem_addr(&bar_dkf[G % C::PD]);
        mbar_expect_tx(dbar, (uint32_t)C::DKR);
        bulk_g2s_plain(dk_base + (uint32_t)((G % C::PD) * C::DKR),
                       reinterpret_cast<const uint8_t*>(p.dk) + ((int64_t)ct * nblk + (int64_t)s * SB) * C::DKB,
                       C::DKS, dbar);
        if (C::FILL) {  // start values of the blocks RT later in this CTA's sequence (past its end: unused)
          int rtf, ctf, sf;
          stage_tile(min(G + C::RT / SB, total_stages - 1), rtf, ctf, sf);
          bulk_g2s_plain(dk_base + (uint32_t)((G % C::PD) * C::DKR + C::DKS),
                         reinterpret_cast<const uint8_t*>(p.fk) + ((int64_t)ctf * nblk + (int64_t)sf * SB) * C::DKB,
                         C::DKS, dbar);
        }
      }
    };
    // the first stages' weights before waiting for the prep kernel (weights do not depend on it)
    const int pre = min(P, total_stages);
    for (int G = 0; G < pre; ++G) issue_weights(G);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int G = 0; G < pre; ++G) issue_acts(G);
    issued = pre;
    for (int G = pre; G < total_stages; ++G) {
      bool ok = true;
      if (lane == 0) ok = mbar_wait(smem_addr(&bar_empty[G % P]), (uint32_t)(((G / P) & 1) ^ 1), kWaitLimit);
      if (lane == 0 && ok && G >= C::PD)
        ok = mbar_wait(smem_addr(&bar_dke[G % C::PD]), (uint32_t)(((G / C::PD) & 1) ^ 1), kWaitLimit);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) *abort_flag = 1;
        break;
      }
      if (aborted()) break;
      issue_weights(G);
      issue_acts(G);
      issued = G + 1;
    }
  } else if (warp == 9) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      // Q4_0 / TQ2_0: the unpacked fields are unsigned (0..15, 0..3). Q4_0: one MMA per accumulator group on a tile
      // that holds the offset -8 in every byte adds -8 * sum(x), N = AG * NT columns at once (the group's
      // accumulators are consecutive in tensor memory, and its units' activation tiles are consecutive rows of one
      // K-major tile); TQ2_0: the accumulators start at 2^23 + 2^22 - sum(x). Q8_0: signed int8 as stored.
      const uint32_t idesc = tc::instr_desc(NT, FMT == 2);
      const uint32_t idesc_off = tc::instr_desc(NT * AG, true);
      // shared-memory descriptors formed once; per MMA only the address field (bytes / 16) advances, which stays
      // below 2^14 because every operand lies inside this CTA's shared memory (< 228 KB)
      const uint64_t adesc0 = tc::smem_desc(a_base), bdesc0 = tc::smem_desc(sbase + C::RAW);
      const uint64_t odesc = tc::smem_desc(off_tile);
      const int total_groups = total_stages * (SU / GU);
      bool ok = mbar_wait(smem_addr(&bar_tinit), 0u, kWaitLimit);
      tc::fence_after();
      for (int g = 0; g < total_groups && ok && !*abort_flag; ++g) {
        const int U0 = g * GU, G = U0 / SU, u0 = U0 - G * SU;
        if (u0 == 0) ok = mbar_wait(smem_addr(&bar_full[G % P]), (uint32_t)((G / P) & 1), kWaitLimit);
        if (ok) ok = mbar_wait(smem_addr(&bar_afull[g % RAG]), (uint32_t)((g / RAG) & 1), kWaitLimit);
        if (!ok) break;
        tc::fence_after();
        const uint64_t bst = bdesc0 + (uint64_t)(((G % P) * C::STAGE + u0 * C::BT) >> 4);
        const uint64_t at = adesc0 + (uint64_t)(((g % RAG) * GU * C::ATILE) >> 4);
#pragma unroll
        for (int i = 0; i < GU; ++i) {
          const int U = U0 + i, B = U / UPB, ub = U - B * UPB;
          if (ub == 0 && B % AG == 0) {  // the first block of an accumulator group: its accumulators are free
            const int a = B / AG;
            ok = mbar_wait(smem_addr(&bar_acce[a % RTG]), (uint32_t)(((a / RTG) & 1) ^ 1), kWaitLimit);
            if (!ok) break;
            tc::fence_after();
            if (FMT == 0)
              tc::mma_i8(tmem + (uint32_t)((B % RT) * NT), odesc, bst + (uint64_t)((i * C::BT) >> 4), idesc_off, 1u);
          }
          // every MMA accumulates: the epilogue left 2^23 + 2^22 (as an integer) in each accumulator it released
          tc::mma_i8(tmem + (uint32_t)((B % RT) * NT), at + (uint64_t)((i * C::ATILE) >> 4),
                     bst + (uint64_t)((i * C::BT) >> 4), idesc, 1u);
          if (ub == UPB - 1 && B % AG == AG - 1) tc::mma_commit(smem_addr(&bar_accf[(B / AG) % RTG]));
        }
        if (!ok) break;
        tc::mma_commit(smem_addr(&bar_aempty[g % RAG]));
        if (u0 + GU == SU) tc::mma_commit(smem_addr(&bar_empty[G % P]));  // the stage's activation tiles are read
        g_issued = g + 1;
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp >= 4) {
    // ---------------- unpack (warps 4-7): thread r = tile row r ----------------
    const int r = t - 128;
    const int sw = r & 7;
    uint8_t* const a_ptr = ws_smem + (a_base - smem_addr(ws_smem));
    const int total_groups = total_stages * (SU / GU);
    uint32_t raw = 0;
    bool ok = true;
    if (FMT == 0) {  // this row of the offset tile (published to the tensor cores with the first group's tile)
      const uint32_t o = 0xF8F8F8F8u;
      uint8_t* ot = ws_smem + (off_tile - smem_addr(ws_smem));
      *reinterpret_cast<uint4*>(ot + tc::core_off(r, 0)) = make_uint4(o, o, o, o);
      *reinterpret_cast<uint4*>(ot + tc::core_off(r, 16)) = make_uint4(o, o, o, o);
    }
    for (int g = 0; g < total_groups; ++g) {
      const int U0 = g * GU, G = U0 / SU, u0 = U0 - G * SU;
      if (u0 == 0) {
        const bool got = __all_sync(0xffffffffu, mbar_wait(smem_addr(&bar_full[G % P]), (uint32_t)((G / P) & 1),
                                                            kWaitLimit));
        if (!got) ok = false;
        if (!got || aborted()) break;
        raw = sbase + (uint32_t)((G % P) * C::STAGE + r * C::RB);
      }
      if (!__all_sync(0xffffffffu, mbar_wait(smem_addr(&bar_aempty[g % RAG]), (uint32_t)(((g / RAG) & 1) ^ 1),
                                              kWaitLimit))) {
        ok = false;
        break;
      }
      uint8_t* at = a_ptr + (g % RAG) * GU * C::ATILE;
      uint4 tq[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
      if (FMT == 1) {  // the group's 4 k-steps are the 4 fields of the same 32 bytes: (block, half) = (u0 / 8, u0 % 8 / 4)
        const int c0 = (u0 >> 3) * 4 + ((u0 & 7) >> 2) * 2;
        tq[0] = lds_v4(raw + (uint32_t)((c0 ^ sw) << 4));
        tq[1] = lds_v4(raw + (uint32_t)(((c0 + 1) ^ sw) << 4));
      }
#pragma unroll
      for (int i = 0; i < GU; ++i) unpack_unit<FMT>(raw, sw, u0 + i, at + i * C::ATILE, r, tq);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic stores -> tensor-core reads
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_addr(&bar_afull[g % RAG]));
        if (u0 + GU == SU) mbar_arrive(smem_addr(&bar_empty[G % P]));  // this warp is done with the stage's weights
      }
    }
    if (!ok && lane == 0) *abort_flag = 1;
  } else {
    // ---------------- epilogue (warps 0-3): thread t = tile row t = tensor-memory lane t ----------------
    constexpr float kMagic = 12582912.0f;  // 2^23 + 2^22
    constexpr int CW = C::CW;
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
    float acc[NT];
#pragma unroll
    for (int c = 0; c < NT; ++c) acc[c] = 0.f;
    // every accumulator starts at 2^23 + 2^22 as an integer: the MMAs add the exact block dot s onto it, so its bits
    // read as an f32 are exactly 2^23 + 2^22 + s (|s| < 2^22) and the conversion costs no instruction
    constexpr uint32_t kMagicBits = 0x4B400000u;
    if constexpr (!C::FILL) {
#pragma unroll 1
      for (int q = 0; q < RT * NT; q += 16) tc::tmem_st16_fill(tmem + lane_base + (uint32_t)q, kMagicBits);
    } else {
      // TQ2_0: the first RT blocks' start values, 2^23 + 2^22 - sum(x), which the prep kernel (the preceding grid)
      // writes: wait for it, stage the RT x NT values through the (not yet used) scale ring with one load per thread,
      // then every thread stores them into its lane
      asm volatile("griddepcontrol.wait;" ::: "memory");
      uint32_t* stg = reinterpret_cast<uint32_t*>(ws_smem + (sc_base - smem_addr(ws_smem)));
      const int e = 2 * t;
      if (e < RT * NT) {
        const int q = e / NT, c = e % NT;
        int rt, ct, s;
        stage_tile(min(q / SB, max(total_stages - 1, 0)), rt, ct, s);
        const int* src = p.fk + ((int64_t)ct * nblk + (int64_t)s * SB + q % SB) * NT + c;
        const int2 w = total_stages > 0 ? __ldg(reinterpret_cast<const int2*>(src)) : make_int2(0, 0);
        *reinterpret_cast<int2*>(stg + e) = w;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
#pragma unroll 1
      for (int q = 0; q < RT * NT; q += 4)
        tc::tmem_st4(tmem + lane_base + (uint32_t)q, *reinterpret_cast<const uint4*>(stg + q));
      asm volatile("bar.sync 1, 128;" ::: "memory");  // the staging area is the scale ring's again
    }
    // this row's block scales of stage G, LA stages ahead, into its own slot of the scale ring
    auto prefetch_scales = [&](int G) {
      if (G < total_stages) {
        int rt, ct, s;
        stage_tile(G, rt, ct, s);
        const int64_t row = (int64_t)rt * 128 + t;
        const bool ok = row < p.N;
        cp_async_ca<C::SBB>(sc_base + (uint32_t)(((G % PS) * 128 + t) * C::SBB),
                            p.ws + (ok ? row : 0) * p.ldws + (int64_t)s * SB, ok);
      }
      cp_async_commit();
    };
#pragma unroll
    for (int G = 0; G < LA; ++G) prefetch_scales(G);
    tc::tmem_wait_st();
    tc::fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_addr(&bar_tinit));
    const int total_agroups = my_tiles * nbt / AG;
    int ep_k = 0, ep_b = 0;  // tile of this CTA's list and block in the tile
    bool ok = true;
    for (int a = 0; a < total_agroups; ++a) {
      const int B0 = a * AG, GB = B0 / SB, j0 = B0 - GB * SB;
      if (j0 == 0) {  // a new stage: row scales LA stages ahead; this stage's column scales have landed
        prefetch_scales(GB + LA);
        cp_async_wait<LA>();
        const bool got = __all_sync(
            0xffffffffu, mbar_wait(smem_addr(&bar_dkf[GB % C::PD]), (uint32_t)((GB / C::PD) & 1), kWaitLimit));
        if (!got) ok = false;
        if (!got || aborted()) break;
      }
      if (!__all_sync(0xffffffffu, mbar_wait(smem_addr(&bar_accf[a % RTG]), (uint32_t)((a / RTG) & 1), kWaitLimit))) {
        ok = false;
        break;
      }
      tc::fence_after();
      // column and row scales by plain loads: the compiler may issue them ahead of the tensor-memory wait
      const uint8_t* dk0 = ws_smem + (dk_base - smem_addr(ws_smem)) + (GB % C::PD) * C::DKR;
      const uint16_t* sc0 = reinterpret_cast<const uint16_t*>(ws_smem + (sc_base - smem_addr(ws_smem)) +
                                                              ((GB % PS) * 128 + t) * C::SBB);
      // The group's accumulators in chunks of CW columns of one block (blocks ascending: the sum order of the
      // reference). Up to 32 columns the loads are software-pipelined: chunk k + 1 is loaded from tensor memory while
      // chunk k is scaled and summed (measured: Q4_0 lm_head at 16 columns 207 -> 201 us).
      constexpr int CPB = NT / CW, CH = AG * CPB;  // chunks per block, per group
      constexpr bool PIPE = NT <= 32;
      if constexpr (PIPE) {
        auto compute_chunk = [&](int j, int c0, const uint32_t(&vk)[CW]) {
          const float4* dxp = reinterpret_cast<const float4*>(dk0 + j * C::DKB);
          const float dw = f16_bits_to_f32(sc0[j]);
          const float2 dw2 = make_float2(dw, dw);
          // Q4_0 / Q8_0: f32(s) * dw in one fma, fl((2^23 + 2^22 + s) * dw - (2^23 + 2^22) * dw): the product
          // 3 * 2^22 * dw of an f16 dw is exact in f32, so the fma rounds s * dw once, as the multiply would
          const float2 mdw2 = make_float2(-kMagic * dw, -kMagic * dw);
  #pragma unroll
          for (int q = 0; q < CW; q += 4) {
            const float4 dx4 = dxp[(c0 + q) / 4];
            const float dxs[4] = {dx4.x, dx4.y, dx4.z, dx4.w};
  #pragma unroll
            for (int e = 0; e < 4; e += 2) {
              const int c = c0 + q + e;
              const float2 fm = make_float2(__uint_as_float(vk[q + e]), __uint_as_float(vk[q + e + 1]));
              const float2 dx2 = make_float2(dxs[e], dxs[e + 1]);
              float2 a2 = make_float2(acc[c], acc[c + 1]);
              if (FMT != 1) {
                a2 = __ffma2_rn(__ffma2_rn(fm, dw2, mdw2), dx2, a2);  // f32(s) * dw * dx
              } else {
                const float2 f = __fadd2_rn(fm, make_float2(-kMagic, -kMagic));  // exact f32(s)
                a2 = __ffma2_rn(__fmul2_rn(dx2, dw2), f, a2);                  // dx * dw * f32(s)
              }
              acc[c] = a2.x;
              acc[c + 1] = a2.y;
            }
          }
        };
        auto load_chunk = [&](int jb, int c0, uint32_t(&dst)[CW]) {
  #pragma unroll
          for (int h = 0; h < CW; h += 16)
            tc::tmem_ld16_nowait(tmem + lane_base + (uint32_t)(((B0 + jb) % RT) * NT + c0 + h),
                                 *reinterpret_cast<uint32_t(*)[16]>(&dst[h]));
        };
        uint32_t v[2][CW];
        auto wait_chunk = [&](uint32_t(&dst)[CW]) {  // the wait names the registers: no use can move above it
          tc::tmem_wait_ld_regs(*reinterpret_cast<uint32_t(*)[16]>(&dst[0]));
#pragma unroll
          for (int h = 16; h < CW; h += 16) tc::regs_ready(*reinterpret_cast<uint32_t(*)[16]>(&dst[h]));
        };
        load_chunk(0, 0, v[0]);
        wait_chunk(v[0]);
#pragma unroll
        for (int k = 0; k < CH; ++k) {
          if (k + 1 < CH) load_chunk((k + 1) / CPB, ((k + 1) % CPB) * CW, v[(k + 1) & 1]);
          compute_chunk(j0 + k / CPB, (k % CPB) * CW, v[k & 1]);
          if (k + 1 < CH) wait_chunk(v[(k + 1) & 1]);
        }
      } else {
        // wide tiles: one chunk at a time, in registers of its own, written out without the helper lambdas (measured:
        // the pipelined form, and the same loop through the lambdas, spill at 64 columns and ran 518 -> 600 us)
#pragma unroll
        for (int jb = 0; jb < AG; ++jb) {
#pragma unroll
          for (int c0 = 0; c0 < NT; c0 += CW) {
            uint32_t v[CW];
#pragma unroll
            for (int h = 0; h < CW; h += 16)
              tc::tmem_ld16_nowait(tmem + lane_base + (uint32_t)(((B0 + jb) % RT) * NT + c0 + h),
                                   *reinterpret_cast<uint32_t(*)[16]>(&v[h]));
            tc::tmem_wait_ld();
            const int j = j0 + jb;
            const float4* dxp = reinterpret_cast<const float4*>(dk0 + j * C::DKB);
            const float dw = f16_bits_to_f32(sc0[j]);
            const float2 dw2 = make_float2(dw, dw);
            const float2 mdw2 = make_float2(-kMagic * dw, -kMagic * dw);
#pragma unroll
            for (int q = 0; q < CW; q += 4) {
              const float4 dx4 = dxp[(c0 + q) / 4];
              const float dxs[4] = {dx4.x, dx4.y, dx4.z, dx4.w};
#pragma unroll
              for (int e = 0; e < 4; e += 2) {
                const int c = c0 + q + e;
                const float2 fm = make_float2(__uint_as_float(v[q + e]), __uint_as_float(v[q + e + 1]));
                const float2 dx2 = make_float2(dxs[e], dxs[e + 1]);
                float2 a2 = make_float2(acc[c], acc[c + 1]);
                if (FMT != 1) {
                  a2 = __ffma2_rn(__ffma2_rn(fm, dw2, mdw2), dx2, a2);  // f32(s) * dw * dx
                } else {
                  const float2 f = __fadd2_rn(fm, make_float2(-kMagic, -kMagic));  // exact f32(s)
                  a2 = __ffma2_rn(__fmul2_rn(dx2, dw2), f, a2);                  // dx * dw * f32(s)
                }
                acc[c] = a2.x;
                acc[c + 1] = a2.y;
              }
            }
          }
        }
      }
      // the group's accumulators start over for their next blocks (RT later): at the constant, or for TQ2_0 at the
      // start values that came with this stage's column scales
#pragma unroll
      for (int jb = 0; jb < AG; ++jb)
#pragma unroll
        for (int h = 0; h < NT; h += 16) {
          const uint32_t ta = tmem + lane_base + (uint32_t)(((B0 + jb) % RT) * NT + h);
          if constexpr (!C::FILL) {
            tc::tmem_st16_fill(ta, kMagicBits);
          } else {  // four columns per store: few registers live next to the NT sums
            const uint4* src = reinterpret_cast<const uint4*>(dk0 + C::DKS + (j0 + jb) * C::DKB + h * 4);
#pragma unroll
            for (int e = 0; e < 16; e += 4) tc::tmem_st4(ta + (uint32_t)e, src[e / 4]);
          }
        }
      tc::tmem_wait_st();
      tc::fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_addr(&bar_acce[a % RTG]));
        if (j0 + AG == SB) mbar_arrive(smem_addr(&bar_dke[GB % C::PD]));  // done with the stage's column scales
      }
      ep_b += AG;
      if (ep_b == nbt) {  // the tile's last block: store its rows of Y (or of its K split's partial sums)
        const int tile = (int)blockIdx.x + ep_k * (int)gridDim.x;
        const int rc = tile / p.ks, kq = tile - rc * p.ks;
        const int rt = rc / p.nct, ct = rc - rt * p.nct;
        const int64_t row = (int64_t)rt * 128 + t;
        const int col0 = ct * NT, ncols = min(NT, p.M - col0);
        if (row < p.N) {
          if (p.ks == 1) {
#pragma unroll
            for (int c = 0; c < NT; ++c)
              if (c < ncols) p.y[(int64_t)(col0 + c) * p.ldy + p.row0 + row] = acc[c];
          } else {
#pragma unroll
            for (int c = 0; c < NT; ++c)
              if (c < ncols) p.part[((int64_t)kq * p.M + col0 + c) * p.N + row] = acc[c];
          }
        }
#pragma unroll
        for (int c = 0; c < NT; ++c) acc[c] = 0.f;
        ep_b = 0;
        ++ep_k;
      }
    }
    if (!ok && lane == 0) *abort_flag = 1;
    cp_async_wait<0>();
  }

  // ---------------- teardown: nothing in flight when the CTA leaves ----------------
  if (warp == 8 && lane == 0) {
    for (int G = max(0, issued - P); G < issued; ++G)
      mbar_wait(smem_addr(&bar_full[G % P]), (uint32_t)((G / P) & 1), kWaitLimit);
    for (int G = max(0, issued - C::PD); G < issued; ++G)
      mbar_wait(smem_addr(&bar_dkf[G % C::PD]), (uint32_t)((G / C::PD) & 1), kWaitLimit);
  }
  if (warp == 9 && lane == 0 && g_issued > 0)
    mbar_wait(smem_addr(&bar_aempty[(g_issued - 1) % RAG]), (uint32_t)(((g_issued - 1) / RAG) & 1), kWaitLimit);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  if (t == 0 && *abort_flag) atomicCAS(&g_device_error, 0, kErrTimeout);
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(C::TCOLS));
}

// ---------------------------------------------------------------------------------------------------------------
// Prep: f32 activations -> MMA activation tiles + column scales dx, quantized with the standalone quantizers' device
// math (identical bytes and scales); optionally also the standard XQ / XD planes (xq_out, xd_out). Columns M ..
// nct*NT-1 are padding: zero tiles, dx = 0 (their accumulators are never stored).
// ---------------------------------------------------------------------------------------------------------------

// q8_0 (Q4_0 and Q8_0 weights): 8 lanes per 32-value block, as b2q_quant_q8_0; a unit is one block.
template <int FMT, int NT>
__global__ void __launch_bounds__(256) tc_prep_q8_0_kernel(const float* __restrict__ x, int64_t ldx, int M, int64_t K,
                                                           int nct, int8_t* __restrict__ xt, float* __restrict__ dk,
                                                           int8_t* __restrict__ xq_out, float* __restrict__ xd_out) {
  pdl_wait_then_trigger();
  const int64_t nblk = K / 32;
  const int64_t total = (int64_t)nct * NT * nblk;
  const int sub = threadIdx.x & 7;
  const int64_t gwarp = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int64_t nwarp = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t base = gwarp * 4; base < total; base += nwarp * 4) {  // warp-uniform bound (shuffles)
    const int64_t g = base + ((threadIdx.x & 31) >> 3);
    const bool ok = g < total;
    const int64_t c = ok ? g / nblk : 0, b = ok ? g % nblk : 0;
    const bool valid = ok && c < M;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (valid) v = *reinterpret_cast<const float4*>(x + c * ldx + b * 32 + sub * 4);
    float d;
    const uint32_t q = q8_0_quant4(v, &d);
    if (ok) {
      const int ct = (int)(c / NT), cl = (int)(c % NT);
      *reinterpret_cast<uint32_t*>(xt + ((int64_t)ct * nblk + b) * (NT * 32) + tc::core_off(cl, sub * 4)) = q;
      const float dx = valid ? q8_0_stored_scale(d) : 0.f;
      if (sub == 0) dk[((int64_t)ct * nblk + b) * NT + cl] = dx;
      if (valid && xq_out) {
        *reinterpret_cast<uint32_t*>(xq_out + c * K + b * 32 + sub * 4) = q;
        if (sub == 0) xd_out[c * nblk + b] = dx;
      }
    }
  }
}

// q8_K (TQ2_0 weights): one warp per 256-value block, as b2q_quant_q8_K; the block is 8 units.
template <int NT>
__global__ void __launch_bounds__(256) tc_prep_q8_K_kernel(const float* __restrict__ x, int64_t ldx, int M, int64_t K,
                                                           int nct, int8_t* __restrict__ xt, float* __restrict__ dk,
                                                           int* __restrict__ fk, int8_t* __restrict__ xq_out,
                                                           float* __restrict__ xd_out) {
  pdl_wait_then_trigger();
  const int64_t nblk = K / 256, nunits = K / 32;
  const int64_t total = (int64_t)nct * NT * nblk;
  const int lane = threadIdx.x & 31;
  const int64_t stride = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t g = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); g < total; g += stride) {
    const int64_t c = g / nblk, b = g % nblk;
    const bool valid = c < M;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (valid) {
      const float* src = x + c * ldx + b * 256 + lane * 8;
      const float4 a = *reinterpret_cast<const float4*>(src);
      const float4 e = *reinterpret_cast<const float4*>(src + 4);
      v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = e.x, v[5] = e.y, v[6] = e.z, v[7] = e.w;
    }
    uint32_t qlo, qhi;
    const float d = q8_K_quant8(v, lane, &qlo, &qhi);
    const int ct = (int)(c / NT), cl = (int)(c % NT);
    const int64_t unit = b * 8 + (lane >> 2);
    *reinterpret_cast<uint2*>(xt + ((int64_t)ct * nunits + unit) * (NT * 32) + tc::core_off(cl, (lane & 3) * 8)) =
        make_uint2(qlo, qhi);
    // the block's sum of quantized values: the GEMM's accumulators start at 2^23 + 2^22 - sum (the crumbs' offset)
    int qs = __dp4a((int)qlo, 0x01010101, __dp4a((int)qhi, 0x01010101, 0));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) qs += __shfl_xor_sync(0xffffffffu, qs, o);
    if (lane == 0) {
      dk[((int64_t)ct * nblk + b) * NT + cl] = valid ? d : 0.f;
      fk[((int64_t)ct * nblk + b) * NT + cl] = 0x4B400000 - qs;
    }
    if (valid && xq_out) {
      *reinterpret_cast<uint2*>(xq_out + c * K + b * 256 + lane * 8) = make_uint2(qlo, qhi);
      if (lane == 0) xd_out[c * nblk + b] = d;
    }
  }
}

// Split-K: Y[m][row0 + n] = the K splits' partial sums added in split order (deterministic)
__global__ void __launch_bounds__(256) tc_splitk_combine_kernel(const float* __restrict__ part, int ks, int64_t M,
                                                                int64_t N, float* __restrict__ y, int64_t ldy,
                                                                int64_t row0) {
  pdl_wait_then_trigger();
  const int64_t total = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / N, n = i - m * N;
    float acc = part[i];
    for (int k = 1; k < ks; ++k) acc += part[(int64_t)k * total + i];
    y[m * ldy + row0 + n] = acc;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------------------------

static int ws_nt(int64_t M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128; }

static int ws_stage_values(int fmt) { return fmt == 0 ? 256 : fmt == 1 ? 512 : 128; }

static size_t align16(size_t n) { return (n + 15) / 16 * 16; }

// K splits for a layer whose tiles (128 rows x NT columns) do not fill the GPU: the fewest that give at least one tile
// per SM, among the divisors of the stage count that leave each split two stages or more (at most 16); 1 when the
// tiles alone fill it.
int gemm_tc_ws_splits(int fmt, int64_t N, int64_t K, int64_t M) {
  if (N <= 0 || K <= 0 || M <= 0 || K % ws_stage_values(fmt)) return 1;
  DeviceInfo di;
  if (device_info(&di) != B2Q_OK) return 1;
  const int NT = ws_nt(M);
  const int64_t tiles = (N + 127) / 128 * ((M + NT - 1) / NT);
  if (tiles >= di.sms) return 1;
  const int64_t stages = K / ws_stage_values(fmt);
  int best = 1;
  for (int d = 2; d <= 16 && stages / d >= 2; ++d) {
    if (stages % d) continue;
    best = d;
    if (tiles * d >= di.sms) break;
  }
  return best;
}

// Workspace bytes of the warp-specialized path (activation tiles, the column scales, for TQ2_0 the accumulators'
// start values, and with ks > 1 K splits the partial sums, each 16-byte aligned), or 0 if the shape does not fit its
// stages (K a whole number of stages: Q4_0 256, TQ2_0 512, Q8_0 128 values).
size_t gemm_tc_ws_bytes(int fmt, int64_t N, int64_t K, int64_t M, int ks) {
  if (K <= 0 || M <= 0 || K % ws_stage_values(fmt)) return 0;
  const int NT = ws_nt(M);
  const int64_t cols = (M + NT - 1) / NT * NT;
  const int64_t nblk = K / (fmt == 1 ? 256 : 32);
  const size_t per_col_blk = align16((size_t)cols * (size_t)nblk * 4);
  const size_t parts = ks > 1 ? align16((size_t)ks * (size_t)M * (size_t)std::max<int64_t>(N, 0) * 4) : 0;
  return align16((size_t)cols * (size_t)K) + per_col_blk * (fmt == 1 ? 2 : 1) + parts;
}

template <int FMT, int NT>
static int launch_ws(const WsParams& wp, const float* x, int64_t ldx, int8_t* xq_out, float* xd_out,
                     cudaStream_t stream, bool pdl) {
  using C = WsCfg<FMT, NT>;
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  // prep
  {
    const int64_t nblk = wp.K / Fmt<FMT>::kBlock;
    const int64_t items = (int64_t)wp.nct * NT * nblk;
    const int64_t per_cta = FMT == 1 ? 8 : 32;  // 256-thread CTAs: 8 warps x (1 q8_K block | 4 q8_0 blocks)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::max<int64_t>(1, std::min<int64_t>((items + per_cta - 1) / per_cta,
                                                                        (int64_t)di.sms * 8)));
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    int8_t* xt = const_cast<int8_t*>(wp.xt);
    float* dk = const_cast<float*>(wp.dk);
    if constexpr (FMT == 1)
      e = cudaLaunchKernelEx(&cfg, tc_prep_q8_K_kernel<NT>, x, ldx, wp.M, wp.K, wp.nct, xt, dk,
                             const_cast<int*>(wp.fk), xq_out, xd_out);
    else
      e = cudaLaunchKernelEx(&cfg, tc_prep_q8_0_kernel<FMT, NT>, x, ldx, wp.M, wp.K, wp.nct, xt, dk, xq_out, xd_out);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(B2Q_ECUDA, "gemm_tc_ws: prep launch failed: %s", cudaGetErrorString(e));
    }
    rc = after_launch("tc_prep");
    if (rc) return rc;
  }
  // GEMM
  auto fn = gemm_tc_ws_kernel<FMT, NT>;
  cudaError_t e = cudaFuncSetAttribute((const void*)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
  if (e != cudaSuccess) return fail(B2Q_ECUDA, "gemm_tc_ws: %s", cudaGetErrorString(e));
  // all of the unified L1 / shared storage as shared memory: otherwise the driver may pick a split that holds one CTA
  // per SM where the occupancy query (and the persistent grid sized from it) counts two
  e = cudaFuncSetAttribute((const void*)fn, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e != cudaSuccess) return fail(B2Q_ECUDA, "gemm_tc_ws: %s", cudaGetErrorString(e));
  // CTAs per SM, computed here: the runtime's occupancy query answers 1 for every kernel that allocates tensor memory
  // (it cannot know how many columns), which would halve this persistent grid. Limits: shared memory (dynamic +
  // static + the per-CTA reservation), registers per SM sub-partition (16K each; a CTA's 10 warps take at most 3 on
  // one), threads, and tensor-memory columns. Too high a count would only queue CTAs, not deadlock them: they do not
  // wait on one another, and an allocation that finds no free columns waits for a finishing CTA.
  int occ = 0;
  {
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, (const void*)fn);
    if (e != cudaSuccess) return fail(B2Q_ECUDA, "gemm_tc_ws: %s", cudaGetErrorString(e));
    int dev = 0, smem_sm = 0, resv = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&resv, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    const int by_smem = smem_sm / (int)(C::SMEM + fa.sharedSizeBytes + (size_t)resv);
    const int warp_regs = (fa.numRegs + 7) / 8 * 8 * 32;
    const int by_regs = 16384 / (3 * warp_regs);
    occ = std::min(std::min(by_smem, by_regs), std::min(2048 / 320, 512 / C::TCOLS));
  }
  if (occ < 1) return fail(B2Q_ECUDA, "gemm_tc_ws: the kernel does not fit an SM");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)std::min<int64_t>(wp.ntiles, (int64_t)di.sms * occ));
  cfg.blockDim = dim3(320);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, fn, wp);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(B2Q_ECUDA, "gemm_tc_ws: launch failed: %s", cudaGetErrorString(e));
  }
  rc = after_launch(FMT == 0 ? "gemm_tc_ws_q4_0" : FMT == 1 ? "gemm_tc_ws_tq2_0" : "gemm_tc_ws_q8_0");
  if (rc || wp.ks == 1) return rc;
  // split-K: the combine, programmatically dependent on the GEMM
  cudaLaunchConfig_t cc = {};
  const int64_t total = (int64_t)wp.M * wp.N;
  cc.gridDim = dim3((unsigned)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, (int64_t)di.sms * 8)));
  cc.blockDim = dim3(256);
  cc.stream = stream;
  cc.attrs = attr;
  cc.numAttrs = 1;
  e = cudaLaunchKernelEx(&cc, tc_splitk_combine_kernel, (const float*)wp.part, wp.ks, (int64_t)wp.M, wp.N, wp.y,
                         wp.ldy, wp.row0);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(B2Q_ECUDA, "gemm_tc_ws: combine launch failed: %s", cudaGetErrorString(e));
  }
  return after_launch("tc_splitk_combine");
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against the driver library)
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static int encode_weight_map(CUtensorMap* map, const uint8_t* wq, int64_t row_bytes, int64_t N, int64_t ldwq) {
  static std::once_flag once;
  static EncodeTiledFn encode = nullptr;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      encode = reinterpret_cast<EncodeTiledFn>(fn);
    else
      cudaGetLastError();
  });
  if (!encode) return fail(B2Q_ECUDA, "gemm_tc_ws: cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)N};
  const cuuint64_t strides[1] = {(cuuint64_t)ldwq};
  const cuuint32_t box[2] = {128, 128};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(wq), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B2Q_ECUDA, "gemm_tc_ws: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return B2Q_OK;
}

// Fused quantize + tensor-core GEMM, warp-specialized (two launches, three with ks > 1 K splits). The caller checked
// gemm_tc_ws_bytes(..., ks) > 0 and workspace_bytes >= it, ks dividing the stage count, a 16-byte aligned workspace,
// weights and x; ws rows contiguous (ldws = K / block).
int launch_gemm_tc_ws(int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws, const float* x, int64_t ldx,
                      int8_t* xq_out, float* xd_out, float* y, int64_t ldy, int64_t row0, int64_t N, int64_t K,
                      int64_t M, int ks, void* workspace, cudaStream_t stream, bool pdl) {
  const int NT = ws_nt(M);
  WsParams wp{};
  const int64_t row_bytes = K / (fmt == 1 ? 256 : 32) * (fmt == 0 ? 16 : fmt == 1 ? 64 : 32);
  const int rc = encode_weight_map(&wp.wmap, wq, row_bytes, N, ldwq);
  if (rc) return rc;
  wp.wq = wq;
  wp.ldwq = ldwq;
  wp.ws = ws;
  wp.ldws = K / (fmt == 1 ? 256 : 32);
  wp.nct = (int)((M + NT - 1) / NT);
  wp.xt = reinterpret_cast<const int8_t*>(workspace);
  wp.dk = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(workspace) +
                                           align16((size_t)wp.nct * NT * (size_t)K));
  wp.fk = reinterpret_cast<const int*>(reinterpret_cast<const uint8_t*>(wp.dk) +
                                       align16((size_t)wp.nct * NT * (size_t)(K / (fmt == 1 ? 256 : 32)) * 4));
  wp.y = y;
  wp.ldy = ldy;
  wp.row0 = row0;
  wp.N = N;
  wp.K = K;
  wp.M = (int)M;
  wp.ks = std::max(1, ks);
  wp.part = wp.ks > 1 ? reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) +
                                                 gemm_tc_ws_bytes(fmt, N, K, M, 1))
                      : nullptr;
  wp.ntiles = (int)((N + 127) / 128) * wp.nct * wp.ks;
#define B2Q_WS_CASE(F, T) \
  if (fmt == F && NT == T) return launch_ws<F, T>(wp, x, ldx, xq_out, xd_out, stream, pdl);
  B2Q_WS_CASE(0, 16) B2Q_WS_CASE(0, 32) B2Q_WS_CASE(0, 64) B2Q_WS_CASE(0, 128)
  B2Q_WS_CASE(1, 16) B2Q_WS_CASE(1, 32) B2Q_WS_CASE(1, 64) B2Q_WS_CASE(1, 128)
  B2Q_WS_CASE(2, 16) B2Q_WS_CASE(2, 32) B2Q_WS_CASE(2, 64) B2Q_WS_CASE(2, 128)
#undef B2Q_WS_CASE
  return fail(B2Q_EINVAL, "gemm_tc_ws: no kernel for fmt %d", fmt);
}

}  // namespace b2q
