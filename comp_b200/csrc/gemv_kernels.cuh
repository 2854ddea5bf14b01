// Q4_0 x q8_0 and TQ2_0 x q8_K decode GEMVs for sm_100a (HBM-bound weight streaming, integer dp4a block dots).
//
// Replaces COMP's Triton kernels q4_0_gemv / tq2_0_gemv (src/komp/kernels.py:48-142). Same results: every int32
// block dot is exact and identical; Y[m][n] = sum over blocks of the per-block f32 product in the reference's
// multiply order (q4_0: f32(s) * dw * dx, kernels.py:93; tq2_0: dx * dw * f32(s), kernels.py:141), summed in a
// fixed (deterministic) order that differs from the reference's, as the reference's own order differs from KURN's.
//
// Schedule (a "chunk" is 16 consecutive quant bytes of one weight row; C = chunks per row = K/32 for Q4_0, K/64 for
// TQ2_0):
//   * One CTA of T = 32*ceil(C/CPT/32) threads works on a group of R consecutive rows at a time; thread t owns chunks
//     t, t+T, ... (CPT of them) of every row. Each CTA takes a contiguous range of row groups (persistent grid).
//   * Weight streaming, "ring" path: the R rows' quant bytes and scale bytes of a group are bulk-copied by the TMA
//     engine (cp.async.bulk, one elected thread) into a ring of S shared-memory stages, each completing on its own
//     mbarrier; S-1 groups are in flight while one is computed, and the first S-1 are issued before the activation
//     prologue so the HBM stream starts at once. Stage release needs no extra barrier: the per-group reduction's
//     __syncthreads orders every read of a stage before it is refilled. Every mbarrier wait is bounded.
//   * "register" path (unaligned scale rows, or the byte-wise variant): 128-bit streaming loads straight into
//     registers, double-buffered one group ahead.
//   * Activations (int8 q8 planes, or f32 quantized in the prologue) are staged once per CTA into shared memory in a
//     permuted layout: for column m, bit-field j and chunk c, the 16 activation bytes that multiply bit-field j of
//     weight chunk c sit at xs[m][j][c] (one conflict-free 128-bit shared load per thread). Q4_0 has j in {lo, hi}
//     nibble; TQ2_0 has j in {crumb 0..3}.
//   * Math per chunk and column: the weight word is masked once per bit-field and dotted with dp4a; the high fields
//     are left in place (u32 x s32 dp4a) and the exact multiple of 2^k is shifted out afterwards, e.g. Q4_0:
//     s = dp4a(w & 0x0F0F0F0F, xl) + (dp4a_u(w & 0xF0F0F0F0, xh) >> 4) - 8 * sum(x). The offsets (-8 for Q4_0,
//     -1 for TQ2_0) are folded in with per-chunk activation sums precomputed in the prologue. TQ2_0 blocks span 4
//     chunks (4 adjacent threads), whose partial dots are combined with two xor-shuffles before scaling.
//   * Per-group reduction: warp shuffles, then a cross-warp sum in shared memory in fixed warp order. The summation
//     order of a row depends only on (K, T, CPT), so Y is bit-identical across paths, variants, R and grid size.
#pragma once

#include "b2q_device.cuh"
#include "b2q_internal.h"

namespace b2q {

constexpr int kMaxThreads = 512;
constexpr int kMaxColumns = 4;  // columns per launch; more are processed in groups of 4 (weights re-read per group)
constexpr int kMaxStages = 8;   // ring stages at most (b2q_set_pipeline)
constexpr long long kWaitLimit = 1LL << 20;  // bounded mbarrier polls (each try_wait also suspends in hardware)
constexpr int kErrTimeout = 1;

// Set by a kernel whose bounded wait gave up; read and cleared by b2q_device_error (gemv_ring.cu, the translation unit
// whose kernels write it; other units including this header hold an unused copy).
static __device__ int g_device_error = 0;

struct GemvParams {
  const uint8_t* wq;
  int64_t ldwq;
  const int16_t* ws;
  const int8_t* xq;       // int8 activations [M][K] (null when x_f32 is given)
  const float* xd;        // activation scales [M][nblk] (null when x_f32 is given)
  const float* x_f32;     // f32 activations [M][ldx] for the fused quantizer prologue, or null
  int64_t ldx;
  int8_t* xq_out;         // fused prologue: CTA 0 also stores the quantized activations here (nullable)
  float* xd_out;
  float* y;               // [M][ldy]; output row index is row0 + local row
  int64_t ldy;
  int64_t row0;
  int32_t* s;             // [M][N][nblk] int32 block dots (nullable)
  // fused all-gather (multi-GPU): own rows go to y; every output value is also sent to each peer's receive buffer as
  // one 8-byte (value, flag) store; each CTA then collects its slice of the peers' rows from its own receive buffer
  unsigned long long* const* rx_peers;  // device array [nranks] of the ranks' receive buffers (peer-mapped), or null
  unsigned long long* rx;  // this rank's receive buffer: 2 parities x rx_stride entries ((m, row) -> m*ldy + row)
  int64_t rx_stride;      // entries per parity
  unsigned long long* done;  // CTAs completed over all calls of this layer (call index = done / gridDim.x)
  int64_t N_total;
  int32_t* status;
  int rank, nranks;
  long long spin_limit;
  int64_t N;              // rows in this launch
  int64_t K;
  int M;                  // columns in this launch (1..kMaxColumns)
  int C;                  // 16-byte chunks per row
  int CPT;                // chunks per thread per row
  int64_t groups;         // ceil(N / R)
  // split-K (gridDim.y = splits): split s handles K columns [s*K, (s+1)*K) of the full rows -- p.K, p.C are the
  // per-split values -- and writes its partial sums to y + s*y_split; strides below refer to the full matrices
  int64_t ldws;           // scale-plane row stride (elements)
  int64_t ldxq;           // int8 activation row stride (bytes); also for xq_out
  int64_t ldxd;           // activation scale row stride (elements); also for xd_out
  int64_t y_split;        // elements between the partial outputs of consecutive splits
  int stages;             // ring path: shared-memory stages
  uint32_t stage_bytes;   // ring path: bytes per stage (R rows of quants, then R rows of scales, 16-byte padded)
  int dense;              // ring path: ldwq == C*16, so a group's quant rows are one contiguous copy
  int cluster;            // ring path, activations in registers: CTAs per cluster sharing the activation prologue
};

template <int FMT>
struct Fmt;
// kQBytes: quant bytes per block; kOffset: the weights' stored offset (value = field - kOffset), folded in as
// -kOffset * sum(x); kActQ80: the activations are q8_0 (32-value blocks, f16-exact scales), else q8_K; kLayout: the
// format whose quant-plane and activation layout this one shares (IQ4_NL is laid out exactly as Q4_0).
// kScaleBytes: bytes of the scale plane per block (an f16 scale, or Q4_K's 20-byte record).
template <>
struct Fmt<0> {  // Q4_0: 32-value blocks, 1 chunk per block, 2 bit-fields (nibbles)
  static constexpr int kBlock = 32, kChunkShift = 0, kFields = 2, kQBytes = 16, kOffset = 8, kLayout = 0;
  static constexpr int kScaleBytes = 2;
  static constexpr bool kActQ80 = true;
};
template <>
struct Fmt<1> {  // TQ2_0: 256-value blocks, 4 chunks per block, 4 bit-fields (crumbs)
  static constexpr int kBlock = 256, kChunkShift = 2, kFields = 4, kQBytes = 64, kOffset = 1, kLayout = 1;
  static constexpr int kScaleBytes = 2;
  static constexpr bool kActQ80 = false;
};
template <>
struct Fmt<2> {  // Q8_0 (an extension beyond the reference: ggml block_q8_0): 32 int8 values, 2 chunks per block
  static constexpr int kBlock = 32, kChunkShift = 1, kFields = 1, kQBytes = 32, kOffset = 0, kLayout = 2;
  static constexpr int kScaleBytes = 2;
  static constexpr bool kActQ80 = true;
};
template <>
struct Fmt<3> {  // IQ4_NL (an extension: ggml block_iq4_nl): Q4_0's layout (kLayout 0), nibbles index 16 int8 levels
  static constexpr int kBlock = 32, kChunkShift = 0, kFields = 2, kQBytes = 16, kOffset = 0, kLayout = 0;
  static constexpr int kScaleBytes = 2;
  static constexpr bool kActQ80 = true;
};
// Q4_K (an extension: ggml block_q4_K) in this backend's split planes: 256-value super-blocks of eight 32-value
// sub-blocks; each 16-byte chunk is one sub-block laid out as a Q4_0 block (kLayout 0: the same activation layout),
// nibbles 0..15 with no offset; the scale plane holds per super-block f16 d, f16 dmin and the bytes (sc_j, m_j).
// Value = d * sc_j * q - dmin * m_j; q8_K activations. The chunk sums (kOffset 1: the plain sum) feed the min term.
template <>
struct Fmt<4> {
  static constexpr int kBlock = 256, kChunkShift = 3, kFields = 2, kQBytes = 128, kOffset = 1, kLayout = 0;
  static constexpr int kScaleBytes = 20;
  static constexpr bool kActQ80 = false;
};

// A weight row's scale for one chunk: the f32 block scale; Q4_K: d, dmin and its sub-block's sc, m.
template <int FMT>
struct RowScale {
  float d;
};
template <>
struct RowScale<4> {
  float d, dmin;
  int sc, mn;
};
// From the block's scale bytes in shared memory (rec: the row's scale plane in the stage, c: the chunk).
template <int FMT>
__device__ __forceinline__ RowScale<FMT> row_scale_smem(uint32_t rec, int c);

// ggml's IQ4_NL levels (kvalues_iq4nl) as little-endian int8 bytes: levels 0-3, 4-7, 8-11, 12-15.
constexpr uint32_t kIq4Lv0 = 0xBFAD9881u, kIq4Lv1 = 0xF6EADDCFu, kIq4Lv2 = 0x26190D01u, kIq4Lv3 = 0x71594535u;

// The levels of the four nibbles in bits 0-15 of `nibs`, as four int8 bytes (nibble j -> byte j): two byte-permute
// lookups, one in each half of the table (index = nibble & 7), and a third that takes each byte from the half its
// nibble's bit 3 selects.
__device__ __forceinline__ uint32_t iq4nl_levels4(uint32_t nibs) {
  const uint32_t lo = __byte_perm(kIq4Lv0, kIq4Lv1, nibs & 0x7777u);
  const uint32_t hi = __byte_perm(kIq4Lv2, kIq4Lv3, nibs & 0x7777u);
  return __byte_perm(lo, hi, 0x3210u | ((nibs >> 1) & 0x4444u));
}

// IQ4_NL activation chunks are kept interleaved the way the lookups order the weight levels: a weight word's low 16
// bits give the levels of values 4k, 16+4k, 4k+1, 16+4k+1 and its high 16 bits those of 4k+2, 16+4k+2, 4k+3,
// 16+4k+3. Field 0 word k = bytes 0, 1 of the natural words k of fields 0 and 1, interleaved; field 1 word k = bytes
// 2, 3. Applied once where a chunk's activations are loaded, so the per-row dot does no permutes of its own.
__device__ __forceinline__ void iq4nl_interleave(uint4 (&x)[4]) {
  const uint4 a = x[0], b = x[1];
  x[0] = make_uint4(__byte_perm(a.x, b.x, 0x5140u), __byte_perm(a.y, b.y, 0x5140u), __byte_perm(a.z, b.z, 0x5140u),
                    __byte_perm(a.w, b.w, 0x5140u));
  x[1] = make_uint4(__byte_perm(a.x, b.x, 0x7362u), __byte_perm(a.y, b.y, 0x7362u), __byte_perm(a.z, b.z, 0x7362u),
                    __byte_perm(a.w, b.w, 0x7362u));
}

// Base pointers of this CTA's K split (blockIdx.y); with one split every offset is zero.
template <int FMT>
struct Split {
  static __device__ __forceinline__ int64_t nblk(const GemvParams& p) { return p.K / Fmt<FMT>::kBlock; }
  static __device__ __forceinline__ const uint8_t* wq(const GemvParams& p) {
    return p.wq + (int64_t)blockIdx.y * (p.K / Fmt<FMT>::kBlock * Fmt<FMT>::kQBytes);
  }
  static __device__ __forceinline__ const int16_t* ws(const GemvParams& p) {
    return p.ws + (int64_t)blockIdx.y * nblk(p) * (Fmt<FMT>::kScaleBytes / 2);
  }
  static __device__ __forceinline__ const int8_t* xq(const GemvParams& p) { return p.xq + (int64_t)blockIdx.y * p.K; }
  static __device__ __forceinline__ const float* xd(const GemvParams& p) { return p.xd + (int64_t)blockIdx.y * nblk(p); }
  static __device__ __forceinline__ const float* xf(const GemvParams& p) {
    return p.x_f32 + (int64_t)blockIdx.y * p.K;
  }
  static __device__ __forceinline__ int8_t* xq_out(const GemvParams& p) {
    return p.xq_out + (int64_t)blockIdx.y * p.K;
  }
  static __device__ __forceinline__ float* xd_out(const GemvParams& p) {
    return p.xd_out + (int64_t)blockIdx.y * nblk(p);
  }
  static __device__ __forceinline__ float* y(const GemvParams& p) { return p.y + (int64_t)blockIdx.y * p.y_split; }
};

// Position (in 16-byte units, within one activation column) of the q-th 16-byte piece of the natural int8 layout.
template <int FMT>
__device__ __forceinline__ int perm_unit(int q, int C) {
  if (Fmt<FMT>::kLayout == 0) return (q & 1) * C + (q >> 1);  // block b = q/2, nibble field h = q%2
  if (FMT == 2) return q;                                       // Q8_0: chunk c holds values 16c .. 16c+15
  const int b = q >> 4, o = q & 15;              // 16 pieces per 256-value block
  const int j = (o >> 1) & 3, c = 2 * (o >> 3) + (o & 1);
  return j * C + 4 * b + c;
}

// ------------------------------------------------------------------------------------------------------------------
// mbarrier / bulk-copy primitives (PTX ISA: mbarrier, cp.async.bulk; sm_90+)
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Bounded wait for the phase with the given parity to complete; false if the limit ran out.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, long long limit) {
  for (long long i = 0; i < limit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Global -> shared bulk copy into this CTA's own shared memory, completion counted in bytes on `bar`; dst, src and
// bytes are multiples of 16. The source is always this GPU's own memory (local weights).
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(pol)
      : "memory");
}


__device__ __forceinline__ uint4 lds_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint16_t lds_u16(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

template <int FMT>
__device__ __forceinline__ RowScale<FMT> row_scale_smem(uint32_t rec, int c) {
  return RowScale<FMT>{f16_bits_to_f32(lds_u16(rec + (uint32_t)(c >> Fmt<FMT>::kChunkShift) * 2u))};
}
template <>
__device__ __forceinline__ RowScale<4> row_scale_smem<4>(uint32_t rec, int c) {
  const uint32_t base = rec + (uint32_t)(c >> 3) * 20u;
  const uint32_t dd = lds_u32(base);                              // f16 d, f16 dmin
  const uint32_t sm = lds_u16(base + 4u + 2u * (uint32_t)(c & 7));  // sc_j, m_j
  return RowScale<4>{f16_bits_to_f32((uint16_t)(dd & 0xffffu)), f16_bits_to_f32((uint16_t)(dd >> 16)),
                     (int)(sm & 0xffu), (int)(sm >> 8)};
}

// ------------------------------------------------------------------------------------------------------------------
// Activation prologue: fills xs (permuted int8), xsum (per-chunk offset correction) and xscale (per-block f32 scale).
// Loads are batched (kUnroll per thread in flight) so the prologue costs a few L2 round trips, not one per item.
// ------------------------------------------------------------------------------------------------------------------
constexpr int kUnroll = 4;

template <int FMT>
__device__ __forceinline__ void stage_activations(const GemvParams& p, uint8_t* xs, int* xsum, float* xscale) {
  const int T = blockDim.x, tt = threadIdx.x;
  const int K = (int)p.K, C = p.C, M = p.M;
  const int nblk = K / Fmt<FMT>::kBlock;
  if (p.x_f32 == nullptr) {
    const int units = K / 16;
    const int total = M * units;
    for (int base = tt; base < total; base += T * kUnroll) {
      uint4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int idx = base + u * T;
        if (idx < total) {
          const int m = idx / units, q = idx - m * units;
          v[u] = *reinterpret_cast<const uint4*>(Split<FMT>::xq(p) + (int64_t)m * p.ldxq + (int64_t)q * 16);
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int idx = base + u * T;
        if (idx < total) {
          const int m = idx / units, q = idx - m * units;
          *reinterpret_cast<uint4*>(xs + (int64_t)m * K + perm_unit<FMT>(q, C) * 16) = v[u];
        }
      }
    }
    for (int idx = tt; idx < M * nblk; idx += T) {
      const int m = idx / nblk, b = idx - m * nblk;
      xscale[idx] = Split<FMT>::xd(p)[(int64_t)m * p.ldxd + b];
    }
  } else if (Fmt<FMT>::kActQ80) {
    // q8_0: 8 lanes per 32-value block (4 blocks per warp per slot); kUnroll slots of loads in flight per lane
    const int lane = tt & 31, sub = lane & 7, nw = T / 32;
    const bool writer = (blockIdx.x == 0) && (p.xq_out != nullptr);
    const int total = M * nblk;
    for (int base = (tt >> 5) * 4; base < total; base += nw * 4 * kUnroll) {
      float4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int g = base + u * nw * 4 + (lane >> 3);
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (g < total) {
          const int m = g / nblk, b = g - m * nblk;
          v[u] = *reinterpret_cast<const float4*>(Split<FMT>::xf(p) + (int64_t)m * p.ldx + b * 32 + sub * 4);
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int g = base + u * nw * 4 + (lane >> 3);
        float d;
        const uint32_t q = q8_0_quant4(v[u], &d);  // whole warp: shuffles inside
        if (g < total) {
          const int m = g / nblk, b = g - m * nblk;
          // Q4_0: low / high nibble fields of block b at xs[field][b]; Q8_0: natural order
          const int pos = Fmt<FMT>::kLayout == 0 ? ((sub >> 2) * C + b) * 16 + (sub & 3) * 4 : b * 32 + sub * 4;
          *reinterpret_cast<uint32_t*>(xs + (int64_t)m * K + pos) = q;
          const float ds = q8_0_stored_scale(d);
          if (sub == 0) xscale[m * nblk + b] = ds;
          if (writer) {
            *reinterpret_cast<uint32_t*>(Split<FMT>::xq_out(p) + (int64_t)m * p.ldxq + b * 32 + sub * 4) = q;
            if (sub == 0 && p.xd_out) Split<FMT>::xd_out(p)[(int64_t)m * p.ldxd + b] = ds;
          }
        }
      }
    }
  } else {
    // q8_K: one warp per 256-value block, lane l holds values 8l..8l+7; kUnroll blocks of loads in flight per warp
    const int lane = tt & 31, nw = T / 32;
    const bool writer = (blockIdx.x == 0) && (p.xq_out != nullptr);
    const int total = M * nblk;
    for (int base = tt >> 5; base < total; base += nw * kUnroll) {
      float4 va[kUnroll], vb[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int g = base + u * nw;
        va[u] = vb[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (g < total) {
          const int m = g / nblk, b = g - m * nblk;
          const float* src = Split<FMT>::xf(p) + (int64_t)m * p.ldx + b * 256 + lane * 8;
          va[u] = *reinterpret_cast<const float4*>(src);
          vb[u] = *reinterpret_cast<const float4*>(src + 4);
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int g = base + u * nw;
        if (g < total) {  // warp-uniform
          const int m = g / nblk, b = g - m * nblk;
          const float v[8] = {va[u].x, va[u].y, va[u].z, va[u].w, vb[u].x, vb[u].y, vb[u].z, vb[u].w};
          uint32_t qlo, qhi;
          const float d = q8_K_quant8(v, lane, &qlo, &qhi);
          const int o = lane >> 1;  // 16-value piece within the block
          // TQ2_0: field (o / 2) % 4 of chunk 4b + 2 (o / 8) + o % 2; Q4_K: field o % 2 of chunk 8b + o / 2
          const int j = FMT == 4 ? (o & 1) : ((o >> 1) & 3);
          const int cc = FMT == 4 ? 8 * b + (o >> 1) : 4 * b + 2 * (o >> 3) + (o & 1);
          *reinterpret_cast<uint2*>(xs + (int64_t)m * K + (j * C + cc) * 16 + (lane & 1) * 8) = make_uint2(qlo, qhi);
          if (lane == 0) xscale[m * nblk + b] = d;
          if (writer) {
            *reinterpret_cast<uint2*>(Split<FMT>::xq_out(p) + (int64_t)m * p.ldxq + b * 256 + lane * 8) =
                make_uint2(qlo, qhi);
            if (lane == 0 && p.xd_out) Split<FMT>::xd_out(p)[(int64_t)m * p.ldxd + b] = d;
          }
        }
      }
    }
  }
  __syncthreads();
  // per-chunk activation sums: Q4_0 8 * (sum of the block's 32 values); TQ2_0 sum of the chunk's 64 values
  for (int idx = tt; idx < M * C; idx += T) {
    const int m = idx / C, c = idx - m * C;
    const uint4* col = reinterpret_cast<const uint4*>(xs + (int64_t)m * K);
    int sum = 0;
#pragma unroll
    for (int j = 0; j < Fmt<FMT>::kFields; ++j) {
      const uint4 v = col[j * C + c];
      sum += bytesum(v.x) + bytesum(v.y) + bytesum(v.z) + bytesum(v.w);
    }
    xsum[idx] = Fmt<FMT>::kOffset * sum;
  }
  __syncthreads();
}

// ------------------------------------------------------------------------------------------------------------------
// Integer block dots of one chunk: weight word w (4 words of 16 bytes) against the activation fields of column m.
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t word_of(const uint4& v, int k) {
  return k == 0 ? v.x : (k == 1 ? v.y : (k == 2 ? v.z : v.w));
}

template <int FMT, bool BYTES>
__device__ __forceinline__ int chunk_dot(const uint4 w, const uint4 (&x)[4], int xsum) {
  if (FMT == 3 && !BYTES) {
    // IQ4_NL: word k holds the nibbles of values 4k..4k+3 (low) and 16+4k..16+4k+3 (high). Table indices and
    // half-selectors are formed once per word (iq4nl_levels4's steps, both halves at once); the lookups give the
    // levels in nibble order, which is the order the activations are kept in (iq4nl_interleave)
    int s = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t wk = word_of(w, k);
      const uint32_t idx = wk & 0x77777777u, sel = 0x32103210u | ((wk >> 1) & 0x44444444u);
      const uint32_t ih = idx >> 16;
      const uint32_t va = __byte_perm(__byte_perm(kIq4Lv0, kIq4Lv1, idx), __byte_perm(kIq4Lv2, kIq4Lv3, idx), sel);
      const uint32_t vb = __byte_perm(__byte_perm(kIq4Lv0, kIq4Lv1, ih), __byte_perm(kIq4Lv2, kIq4Lv3, ih), sel >> 16);
      s = __dp4a((int)va, (int)word_of(x[0], k), s);
      s = __dp4a((int)vb, (int)word_of(x[1], k), s);
    }
    return s;
  }
  if (FMT == 2 && !BYTES) {  // Q8_0: signed weights, no field extraction and no offset
    int s = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) s = dp4a_ss((int)word_of(w, k), (int)word_of(x[0], k), s);
    return s;
  }
  if (!BYTES) {
#ifndef B2Q_DP4A_SIGNED_ONLY
    if (FMT == 0) {
      int lo = 0, hi = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t wk = word_of(w, k);
        lo = dp4a_ss((int)(wk & 0x0F0F0F0Fu), (int)word_of(x[0], k), lo);
        hi = dp4a_us(wk & 0xF0F0F0F0u, (int)word_of(x[1], k), hi);
      }
      return lo + (hi >> 4) - xsum;
    } else {
      int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t wk = word_of(w, k);
        a0 = dp4a_us(wk & 0x03030303u, (int)word_of(x[0], k), a0);
        a1 = dp4a_us(wk & 0x0C0C0C0Cu, (int)word_of(x[1], k), a1);
        a2 = dp4a_us(wk & 0x30303030u, (int)word_of(x[2], k), a2);
        a3 = dp4a_us(wk & 0xC0C0C0C0u, (int)word_of(x[3], k), a3);
      }
      return a0 + (a1 >> 2) + (a2 >> 4) + (a3 >> 6) - xsum;
    }
#else
    // Alternative (B2Q_DP4A_SIGNED_ONLY): signed dp4a only, every weight byte kept below 128: fields at the same power-of-two scale share one
    // accumulator, and the scale is removed by an exact arithmetic shift at the end.
    if (FMT == 0) {
      // low nibbles (values i) and high nibbles shifted down (values 16+i) both at 1x: one accumulator
      int acc = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t wk = word_of(w, k);
        acc = dp4a_ss((int)(wk & 0x0F0F0F0Fu), (int)word_of(x[0], k), acc);
        acc = dp4a_ss((int)((wk >> 4) & 0x0F0F0F0Fu), (int)word_of(x[1], k), acc);
      }
      return acc - xsum;
    } else {
      // crumbs 0 and 1 at 1x (w and w>>2 masked with 0x03), crumbs 2 and 3 at 16x (masked with 0x30)
      int a01 = 0, a23 = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t wk = word_of(w, k), wh = wk >> 2;
        a01 = dp4a_ss((int)(wk & 0x03030303u), (int)word_of(x[0], k), a01);
        a01 = dp4a_ss((int)(wh & 0x03030303u), (int)word_of(x[1], k), a01);
        a23 = dp4a_ss((int)(wk & 0x30303030u), (int)word_of(x[2], k), a23);
        a23 = dp4a_ss((int)(wh & 0x30303030u), (int)word_of(x[3], k), a23);
      }
      return a01 + (a23 >> 4) - xsum;
    }
#endif
  } else {
    // byte-wise variant (the reference's MODE 0): every value unpacked to an int32, no offset correction needed
    int s = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t wk = word_of(w, k);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int wb = (int)((wk >> (8 * t)) & 0xffu);
#pragma unroll
        for (int j = 0; j < Fmt<FMT>::kFields; ++j) {
          // IQ4_NL chunks are interleaved (iq4nl_interleave): natural field j, byte t sits in word k of field t/2,
          // byte 2 * (t % 2) + j
          const int xb = FMT == 3 ? (int)(int8_t)((word_of(x[t >> 1], k) >> (8 * (2 * (t & 1) + j))) & 0xffu)
                                  : (int)(int8_t)((word_of(x[j], k) >> (8 * t)) & 0xffu);
          const int val = (FMT == 3)   ? (int)(int8_t)(iq4nl_levels4((wb >> (4 * j)) & 15) & 0xffu)
                          : (FMT == 0) ? ((wb >> (4 * j)) & 15) - 8
                          : (FMT == 1) ? ((wb >> (2 * j)) & 3) - 1
                                       : (int)(int8_t)wb;
          s += val * xb;
        }
      }
    }
    return s;
  }
}


// ------------------------------------------------------------------------------------------------------------------
// Activations of one chunk and column: the kFields 16-byte fields, the offset correction and the block scale.
// ------------------------------------------------------------------------------------------------------------------
struct XChunk {
  uint4 x[4];
  int sum;
  float dx;
};

template <int FMT>
__device__ __forceinline__ void load_xchunk(const GemvParams& p, const uint8_t* xs, const int* xsum,
                                            const float* xscale, int m, int c, bool valid, XChunk& o) {
  const int nblk = (int)(p.K / Fmt<FMT>::kBlock);
  if (valid) {
    const uint4* col = reinterpret_cast<const uint4*>(xs + (int64_t)m * p.K);
#pragma unroll
    for (int j = 0; j < Fmt<FMT>::kFields; ++j) o.x[j] = col[j * p.C + c];
    if (FMT == 3) iq4nl_interleave(o.x);
    o.sum = xsum[m * p.C + c];
    o.dx = xscale[m * nblk + (c >> Fmt<FMT>::kChunkShift)];
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) o.x[j] = make_uint4(0u, 0u, 0u, 0u);
    o.sum = 0;
    o.dx = 0.f;
  }
}

// One chunk c of R rows (weights w[r], scales dw[r]) against MC columns: block dots, S store, f32 accumulation into
// acc[r*MC + m]. Columns m >= p.M are skipped (uniformly). No predicate guards the accumulation: a chunk past the row
// end has zero weights, zero activations and zero scales, and rows past N are never stored.
//   Q4_0 (one block per chunk): acc += f32(s) * dw * dx, the reference's per-block product (kernels.py:93).
//   TQ2_0 (a block spans 4 chunks on 4 adjacent threads): each thread adds its own chunk's exact partial dot,
//     acc += (dx * dw) * f32(s_chunk) (the reference's dx * dw * s order, kernels.py:141, applied per quarter block),
//     so the 4 threads need no exchange; with STORE the exact block dot is assembled with two xor-shuffles for S.
//   Q4_K (a super-block spans 8 chunks): s = the sub-block's exact dot (nibbles 0..15), S = sc * s and the min term
//     M = m * sum(x) as exact ints, acc += dx * (d * f32(S) - dmin * f32(M)); S is what the block dot dump adds up.
template <int FMT, int R, int MC, bool BYTES, bool STORE>
__device__ __forceinline__ void compute_chunk(const GemvParams& p, int64_t g, int c, bool valid, const uint4 (&w)[R],
                                              const RowScale<FMT> (&rs)[R], const XChunk (&xc)[MC],
                                              float (&acc)[R * MC]) {
  const int nblk = (int)(p.K / Fmt<FMT>::kBlock);
  const int blk = c >> Fmt<FMT>::kChunkShift;
#pragma unroll
  for (int m = 0; m < MC; ++m) {
    if (MC == 1 || m < p.M) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        int s;
        if constexpr (FMT == 4) {
          int lo = 0, hi = 0;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t wk = word_of(w[r], k);
            lo = dp4a_ss((int)(wk & 0x0F0F0F0Fu), (int)word_of(xc[m].x[0], k), lo);
            hi = dp4a_us(wk & 0xF0F0F0F0u, (int)word_of(xc[m].x[1], k), hi);
          }
          s = rs[r].sc * (lo + (hi >> 4));
          const float t = __fsub_rn(__fmul_rn(rs[r].d, (float)s), __fmul_rn(rs[r].dmin, (float)(rs[r].mn * xc[m].sum)));
          acc[r * MC + m] = __fmaf_rn(xc[m].dx, t, acc[r * MC + m]);
        } else {
          s = chunk_dot<FMT, BYTES>(w[r], xc[m].x, xc[m].sum);
          if (FMT != 1)  // Q4_0, Q8_0: f32(s) * dw * dx
            acc[r * MC + m] = __fmaf_rn(__fmul_rn((float)s, rs[r].d), xc[m].dx, acc[r * MC + m]);
          else  // TQ2_0: dx * dw * f32(s)
            acc[r * MC + m] = __fmaf_rn(__fmul_rn(xc[m].dx, rs[r].d), (float)s, acc[r * MC + m]);
        }
        if (STORE) {  // the block dot: the partial dots of the block's chunks (adjacent lanes) added up
          int sb = s;
#pragma unroll
          for (int sh = 0; sh < Fmt<FMT>::kChunkShift; ++sh) sb += __shfl_xor_sync(0xffffffffu, sb, 1 << sh);
          const int64_t row = g * R + r;
          const bool first = (c & ((1 << Fmt<FMT>::kChunkShift) - 1)) == 0;
          if (valid && first && row < p.N) p.s[((int64_t)m * p.N + row) * nblk + blk] = sb;
        }
      }
    }
  }
}

// Warp sum of V values per lane (V a power of two <= 32) with V + 4 - log2(V) shuffles instead of 5V: each xor step
// halves the values a lane carries (a reduce-scatter) until one is left, then plain xor steps finish it. Lane l ends
// with the full warp sum of value index l / (32/V). Every value is summed over the xor-16, 8, 4, 2, 1 pairings in the
// same order as a plain xor-tree reduction, so the result is bit-identical to reducing each value separately.
template <int V>
__device__ __forceinline__ float warp_sum_scatter(float (&v)[V], int lane) {
  int off = 16;
#pragma unroll
  for (int n = V; n > 1; n >>= 1) {
    const bool up = (lane & off) != 0;
#pragma unroll
    for (int k = 0; k < n / 2; ++k) {
      const float send = up ? v[k] : v[k + n / 2];
      const float keep = up ? v[k + n / 2] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
    off >>= 1;
  }
  float s = v[0];
#pragma unroll
  for (; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  return s;
}

// Fused all-gather entries: one naturally aligned 64-bit word, flag (1) in the high half, the f32 value's bits in the
// low half, written and read as 64-bit scalars (relaxed, system scope), so the pair is single-copy atomic.
__device__ __forceinline__ unsigned long long rx_word(float v) {
  return (1ull << 32) | (unsigned long long)__float_as_uint(v);
}
__device__ __forceinline__ void rx_store(unsigned long long* dst, unsigned long long w) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(dst), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long rx_load(const unsigned long long* src) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(src) : "memory");
  return w;
}

// Group reduction: warp reduce-scatter, cross-warp sum in fixed warp order, store of R x M outputs. Contains one
// __syncthreads. red is double-buffered so the next group's writes never race this group's reads.
template <int R, int MC>
__device__ __forceinline__ void reduce_store(const GemvParams& p, int64_t g, float (&acc)[R * MC], float* red,
                                             int buf, int parity, int sum_warp = 0) {
  constexpr int V = R * MC;
  const int nwarps = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float s = warp_sum_scatter<V>(acc, lane);
#pragma unroll
  for (int k = 0; k < V; ++k) acc[k] = 0.f;
  if ((lane & (32 / V - 1)) == 0) red[(buf * nwarps + warp) * V + lane / (32 / V)] = s;
  __syncthreads();
  if (warp == sum_warp && lane < V) {  // the cross-warp sum of this group is done by warp sum_warp
    const int r = lane / MC, m = lane - r * MC;
    const int64_t row = g * R + r;
    if (m < p.M && row < p.N) {
      float v = 0.f;
      for (int w = 0; w < nwarps; ++w) v += red[(buf * nwarps + w) * V + lane];
      const int64_t idx = (int64_t)m * p.ldy + p.row0 + row;
      p.y[idx + (int64_t)blockIdx.y * p.y_split] = v;
      if (p.rx_peers != nullptr) {  // fused all-gather: (value, flag 1) into every other rank's receive buffer
        const int64_t off = (int64_t)parity * p.rx_stride + idx;
        const unsigned long long word = rx_word(v);
        for (int q = 0; q < p.nranks; ++q)
          if (q != p.rank) rx_store(p.rx_peers[q] + off, word);
      }
    }
  }
}

// Fused all-gather, receive side. Every value a peer sends is one naturally aligned 64-bit scalar store of the word
// (flag << 32 | value bits); a 64-bit scalar access is single-copy atomic, so a reader that sees the flag also sees
// the value, and no fence is needed. Each CTA collects a contiguous slice of the
// entries of the peers' rows: it polls each entry (bounded) until the flag is set, copies the value into y and clears
// the flag for the call after next. The receive buffer alternates between two parities per call, so a fast peer's
// next call never overwrites entries of this call that are still unread: a rank starts call t+2 only after it has
// received every rank's rows of call t+1, which each rank sends after finishing call t.
// Call index (and so the parity) of this launch: every CTA of a call reads done / gridDim.x at its start, which is
// exact because only CTAs of this call can have incremented it since the previous call completed.
__device__ __forceinline__ int call_parity(const GemvParams& p) {
  if (p.rx_peers == nullptr) return 0;
  const unsigned long long d = *reinterpret_cast<volatile unsigned long long*>(p.done);
  return (int)((d / gridDim.x) & 1ull);
}

__device__ __forceinline__ void allgather_collect(const GemvParams& p, int parity) {
  const int64_t peer_rows = p.N_total - p.N;
  const int64_t total = (int64_t)p.M * peer_rows;
  const int64_t e_begin = (total * blockIdx.x) / gridDim.x, e_end = (total * (blockIdx.x + 1)) / gridDim.x;
  unsigned long long* rx = p.rx + (int64_t)parity * p.rx_stride;
  int err = 0;
  for (int64_t e = e_begin + threadIdx.x; e < e_end; e += blockDim.x) {
    const int64_t m = e / peer_rows, r = e - m * peer_rows;
    const int64_t row = r < p.row0 ? r : r + p.N;
    const int64_t idx = m * p.ldy + row;
    unsigned long long* src = rx + idx;
    // after a timeout the thread stops polling but still clears the rest of its entries, so values that arrived
    // in time are not left flagged for a later call of the same parity
    long long spins = 0;
    while (!err) {
      const unsigned long long word = rx_load(src);
      if ((word >> 32) != 0ull) {
        p.y[idx] = __uint_as_float((uint32_t)word);
        break;
      }
      if (++spins > p.spin_limit) err = 1;
    }
    rx_store(src, 0ull);
  }
  if (err && p.status) atomicExch(p.status, 1);
  __syncthreads();
  if (threadIdx.x == 0) atomicAdd(p.done, 1ull);
}

// ------------------------------------------------------------------------------------------------------------------
// Register path: weights streamed straight into registers, double-buffered one unit (group, chunk round) ahead.
// XREG (one column, one chunk per thread): the thread's activation chunk stays in registers for the whole kernel;
// otherwise activations are read from shared memory per chunk.
// ------------------------------------------------------------------------------------------------------------------
template <int R>
struct WeightRegs {
  uint4 w[R];
  uint16_t sc[R];
};

template <int FMT, int R>
__device__ __forceinline__ void load_unit(const GemvParams& p, int64_t g, int i, bool active, WeightRegs<R>& u) {
  const int c = (int)threadIdx.x + i * (int)blockDim.x;
  const int nblk = (int)(p.K / Fmt<FMT>::kBlock);
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int64_t row = g * R + r;
    if (active && c < p.C && row < p.N) {
      u.w[r] = ld_stream_v4(Split<FMT>::wq(p) + row * p.ldwq + (int64_t)c * 16);
      u.sc[r] = ld_stream_u16(Split<FMT>::ws(p) + row * p.ldws + (c >> Fmt<FMT>::kChunkShift));
    } else {
      u.w[r] = make_uint4(0u, 0u, 0u, 0u);
      u.sc[r] = 0;
    }
  }
}

// XREG prologue: this thread's activation chunk straight from global memory into registers -- no shared memory and
// no CTA barrier. int8 input: the chunk's q8 bytes, offset sum and scale. f32 input: the chunk is quantized here with
// the math of b2q_quant_q8_0 / b2q_quant_q8_K: a Q4_0 chunk is a whole q8_0 block (one thread); a TQ2_0 chunk is a
// quarter of a q8_K block, whose largest magnitude, its first index and its signed value are combined over the 4
// threads of the block by xor-shuffles (all lanes of the warp take part; chunks past the row end are zero).
// CTA 0 also stores the quantized activations when xq_out is given.
template <int FMT>
__device__ __forceinline__ void load_x_direct(const GemvParams& p, int c, bool valid, XChunk& o, int m = 0) {
#pragma unroll
  for (int j = 0; j < 4; ++j) o.x[j] = make_uint4(0u, 0u, 0u, 0u);
  o.sum = 0;
  o.dx = 0.f;
  // the first CTA (with clusters: the first cluster's CTAs, each for the chunks it quantizes) writes XQ/XD out
  const bool writer = (blockIdx.x < (unsigned)max(1, p.cluster)) && (p.xq_out != nullptr) && valid;
  if (p.x_f32 == nullptr) {
    if (!valid) return;
    if (Fmt<FMT>::kLayout == 0) {
      const uint4* src = reinterpret_cast<const uint4*>((Split<FMT>::xq(p) + (int64_t)m * p.ldxq) + (int64_t)c * 32);
      o.x[0] = src[0];
      o.x[1] = src[1];
      o.dx = (Split<FMT>::xd(p) + (int64_t)m * p.ldxd)[c >> Fmt<FMT>::kChunkShift];
      if (FMT == 3) {  // no offset term; the chunk interleaved for the level lookups
        iq4nl_interleave(o.x);
        return;
      }
    } else if (FMT == 2) {
      o.x[0] = *reinterpret_cast<const uint4*>((Split<FMT>::xq(p) + (int64_t)m * p.ldxq) + (int64_t)c * 16);
      o.dx = (Split<FMT>::xd(p) + (int64_t)m * p.ldxd)[c >> 1];
    } else {
      const int b = c >> 2, cc = c & 3;
      const int8_t* base = (Split<FMT>::xq(p) + (int64_t)m * p.ldxq) + (int64_t)b * 256 + (cc >> 1) * 128 + (cc & 1) * 16;
#pragma unroll
      for (int j = 0; j < 4; ++j) o.x[j] = *reinterpret_cast<const uint4*>(base + j * 32);
      o.dx = (Split<FMT>::xd(p) + (int64_t)m * p.ldxd)[b];
    }
    int sum = 0;
#pragma unroll
    for (int j = 0; j < Fmt<FMT>::kFields; ++j)
      sum += bytesum(o.x[j].x) + bytesum(o.x[j].y) + bytesum(o.x[j].z) + bytesum(o.x[j].w);
    o.sum = Fmt<FMT>::kOffset * sum;
    return;
  }
  if (FMT == 2) {
    // q8_0 for Q8_0 weights: chunk c holds values 16c .. 16c+15, the block's other half is on lane c ^ 1. Same
    // arithmetic as the q8_0 quantizer (amax / 127, roundf(x * id) from the unrounded d, f16-exact stored scale).
    float4 v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      v[i] = valid ? reinterpret_cast<const float4*>((Split<FMT>::xf(p) + (int64_t)m * p.ldx) + (int64_t)c * 16)[i]
                   : make_float4(0.f, 0.f, 0.f, 0.f);
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int q0 = (int)roundf(__fmul_rn(v[i].x, id)), q1 = (int)roundf(__fmul_rn(v[i].y, id));
      const int q2 = (int)roundf(__fmul_rn(v[i].z, id)), q3 = (int)roundf(__fmul_rn(v[i].w, id));
      w[i] = (uint32_t)(q0 & 0xff) | ((uint32_t)(q1 & 0xff) << 8) | ((uint32_t)(q2 & 0xff) << 16) |
             ((uint32_t)(q3 & 0xff) << 24);
    }
    if (!valid) return;
    o.x[0] = make_uint4(w[0], w[1], w[2], w[3]);
    o.dx = q8_0_stored_scale(d);
    if (writer) {
      *reinterpret_cast<uint4*>((Split<FMT>::xq_out(p) + (int64_t)m * p.ldxq) + (int64_t)c * 16) = o.x[0];
      if ((c & 1) == 0 && p.xd_out) (Split<FMT>::xd_out(p) + (int64_t)m * p.ldxd)[c >> 1] = o.dx;
    }
    return;
  }
  if (FMT == 4) {
    // q8_K for Q4_K: chunk c holds values 32c .. 32c+31 (fields: the first and last 16); the 256-value block spans
    // the 8 chunks (threads) c & ~7 .. c | 7, so the block's signed maximum and minimum, and on a tie between signs
    // the lowest index, are combined over those 8 threads by xor-shuffles (all lanes of the warp take part). Same
    // arithmetic as the q8_K quantizer and the TQ2_0 prologue.
    float v[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 f = valid ? *reinterpret_cast<const float4*>((Split<FMT>::xf(p) + (int64_t)m * p.ldx) + (int64_t)c * 32 + 4 * i)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
      v[4 * i] = f.x, v[4 * i + 1] = f.y, v[4 * i + 2] = f.z, v[4 * i + 3] = f.w;
    }
    float mx8[8], mn8[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      mx8[t] = fmaxf(fmaxf(v[t], v[t + 8]), fmaxf(v[t + 16], v[t + 24]));
      mn8[t] = fminf(fminf(v[t], v[t + 8]), fminf(v[t + 16], v[t + 24]));
    }
#pragma unroll
    for (int n = 4; n >= 1; n >>= 1)
#pragma unroll
      for (int t = 0; t < n; ++t) {
        mx8[t] = fmaxf(mx8[t], mx8[t + n]);
        mn8[t] = fminf(mn8[t], mn8[t + n]);
      }
    float mx = mx8[0], mn = mn8[0];
#pragma unroll
    for (int off = 1; off <= 4; off <<= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
    }
    const float amax = fmaxf(fmaxf(mx, -mn), 0.0f);  // 0 for an all-zero (or all-NaN) block
    float cand = mx >= -mn ? mx : mn;
    const bool tie = mx == -mn && amax != 0.0f;
    if (__any_sync(0xffffffffu, tie)) {
      const int vb = (c & 7) * 32;  // this chunk's first value index within the block
      int key8[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        key8[t] = 0x7fffffff;
#pragma unroll
        for (int j = 3; j >= 0; --j)  // value t + 8j: lower j = lower index, it overrides
          if (fabsf(v[t + 8 * j]) == amax)
            key8[t] = ((vb + t + 8 * j) << 1) | (int)(__float_as_uint(v[t + 8 * j]) >> 31);
      }
#pragma unroll
      for (int n = 4; n >= 1; n >>= 1)
#pragma unroll
        for (int t = 0; t < n; ++t) key8[t] = min(key8[t], key8[t + n]);
      int key = key8[0];
#pragma unroll
      for (int off = 1; off <= 4; off <<= 1) key = min(key, __shfl_xor_sync(0xffffffffu, key, off));
      if (tie) cand = (key & 1) ? -amax : amax;
    }
    const bool nz = amax != 0.0f;
    const float iscale = __fdiv_rn(-127.0f, nz ? cand : 1.0f);
    const float2 is2 = make_float2(iscale, iscale), mg2 = make_float2(12582912.0f, 12582912.0f);
    uint32_t w[8];
    int sum = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float2 p01 = __fmul2_rn(make_float2(v[4 * k], v[4 * k + 1]), is2);
      float2 p23 = __fmul2_rn(make_float2(v[4 * k + 2], v[4 * k + 3]), is2);
      p01 = __fadd2_rn(make_float2(fminf(p01.x, 127.0f), fminf(p01.y, 127.0f)), mg2);
      p23 = __fadd2_rn(make_float2(fminf(p23.x, 127.0f), fminf(p23.y, 127.0f)), mg2);
      w[k] = nz ? pack_low_bytes(__float_as_uint(p01.x), __float_as_uint(p01.y), __float_as_uint(p23.x),
                                 __float_as_uint(p23.y))
                : 0u;
      sum = __dp4a((int)w[k], 0x01010101, sum);
    }
    if (!valid) return;
    o.x[0] = make_uint4(w[0], w[1], w[2], w[3]);  // values 32c .. 32c+15
    o.x[1] = make_uint4(w[4], w[5], w[6], w[7]);  // values 32c+16 .. 32c+31
    o.sum = sum;
    o.dx = nz ? __fdiv_rn(1.0f, iscale) : 0.0f;
    if (writer) {
      uint4* dst = reinterpret_cast<uint4*>((Split<FMT>::xq_out(p) + (int64_t)m * p.ldxq) + (int64_t)c * 32);
      dst[0] = o.x[0];
      dst[1] = o.x[1];
      if ((c & 7) == 0 && p.xd_out) (Split<FMT>::xd_out(p) + (int64_t)m * p.ldxd)[c >> 3] = o.dx;
    }
    return;
  }
  if (Fmt<FMT>::kLayout == 0) {
    if (!valid) return;
    const float4* src = reinterpret_cast<const float4*>((Split<FMT>::xf(p) + (int64_t)m * p.ldx) + (int64_t)c * 32);
    float4 v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = src[i];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
    uint32_t w[8];
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int q0 = (int)roundf(__fmul_rn(v[i].x, id)), q1 = (int)roundf(__fmul_rn(v[i].y, id));
      const int q2 = (int)roundf(__fmul_rn(v[i].z, id)), q3 = (int)roundf(__fmul_rn(v[i].w, id));
      w[i] = (uint32_t)(q0 & 0xff) | ((uint32_t)(q1 & 0xff) << 8) | ((uint32_t)(q2 & 0xff) << 16) |
             ((uint32_t)(q3 & 0xff) << 24);
      sum += q0 + q1 + q2 + q3;
    }
    o.x[0] = make_uint4(w[0], w[1], w[2], w[3]);  // values 0..15 (low-nibble field)
    o.x[1] = make_uint4(w[4], w[5], w[6], w[7]);  // values 16..31 (high-nibble field)
    o.sum = Fmt<FMT>::kOffset * sum;
    o.dx = q8_0_stored_scale(d);
    if (writer) {
      uint4* dst = reinterpret_cast<uint4*>((Split<FMT>::xq_out(p) + (int64_t)m * p.ldxq) + (int64_t)c * 32);
      dst[0] = o.x[0];
      dst[1] = o.x[1];
      if (p.xd_out) (Split<FMT>::xd_out(p) + (int64_t)m * p.ldxd)[c] = o.dx;
    }
    if (FMT == 3) iq4nl_interleave(o.x);  // after the natural-order XQ write-out
    return;
  }
  // TQ2_0 / q8_K: field j of chunk c holds block values (cc/2)*128 + j*32 + (cc%2)*16 + t, t = 0..15
  const int b = c >> 2, cc = c & 3;
  const int vbase = (cc >> 1) * 128 + (cc & 1) * 16;
  float v[4][16];
  if (valid) {
    const float* base = (Split<FMT>::xf(p) + (int64_t)m * p.ldx) + (int64_t)b * 256 + vbase;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int t4 = 0; t4 < 4; ++t4) {
        const float4 f = *reinterpret_cast<const float4*>(base + j * 32 + t4 * 4);
        v[j][t4 * 4 + 0] = f.x, v[j][t4 * 4 + 1] = f.y, v[j][t4 * 4 + 2] = f.z, v[j][t4 * 4 + 3] = f.w;
      }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int t = 0; t < 16; ++t) v[j][t] = 0.f;
  }
  // Signed maximum and minimum of the chunk (balanced trees; fmaxf / fminf ignore NaN), then of the block over its
  // 4 threads. The quantizer divides by the signed value of largest magnitude, the first one on ties (ggml scans
  // with a strict >): when one sign alone reaches the largest magnitude that value is the maximum or the minimum;
  // when both signs reach it, the lower index decides -- an exact search, run only by warps that hold such a block.
  float mx16[16], mn16[16];
#pragma unroll
  for (int t = 0; t < 16; ++t) {
    mx16[t] = fmaxf(fmaxf(v[0][t], v[1][t]), fmaxf(v[2][t], v[3][t]));
    mn16[t] = fminf(fminf(v[0][t], v[1][t]), fminf(v[2][t], v[3][t]));
  }
#pragma unroll
  for (int n = 8; n >= 1; n >>= 1)
#pragma unroll
    for (int t = 0; t < n; ++t) {
      mx16[t] = fmaxf(mx16[t], mx16[t + n]);
      mn16[t] = fminf(mn16[t], mn16[t + n]);
    }
  float mx = mx16[0], mn = mn16[0];
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
  }
  const float amax = fmaxf(fmaxf(mx, -mn), 0.0f);  // 0 for an all-zero (or all-NaN) block
  float cand = mx >= -mn ? mx : mn;
  const bool tie = mx == -mn && amax != 0.0f;
  if (__any_sync(0xffffffffu, tie)) {
    // the lowest value index whose magnitude is amax, with its sign bit: key = index * 2 + sign, minimum over the
    // chunk (a tree) and over the block's 4 threads
    int key16[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      key16[t] = 0x7fffffff;
#pragma unroll
      for (int j = 3; j >= 0; --j)  // lower field = lower index: it overrides
        if (fabsf(v[j][t]) == amax) key16[t] = ((vbase + j * 32 + t) << 1) | (int)(__float_as_uint(v[j][t]) >> 31);
    }
#pragma unroll
    for (int n = 8; n >= 1; n >>= 1)
#pragma unroll
      for (int t = 0; t < n; ++t) key16[t] = min(key16[t], key16[t + n]);
    int key = key16[0];
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) key = min(key, __shfl_xor_sync(0xffffffffu, key, off));
    if (tie) cand = (key & 1) ? -amax : amax;
  }
  const bool nz = amax != 0.0f;
  const float iscale = __fdiv_rn(-127.0f, nz ? cand : 1.0f);
  // q = min(127, rint(iscale * x)) through q8_K_bits' exact add (no conversion unit), two values per packed f32x2
  // multiply and add (each lane rounded as the scalar operation), bytes packed with prmt, summed with dp4a
  const float2 is2 = make_float2(iscale, iscale), mg2 = make_float2(12582912.0f, 12582912.0f);
  int sum = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 p01 = __fmul2_rn(make_float2(v[j][k * 4 + 0], v[j][k * 4 + 1]), is2);
      float2 p23 = __fmul2_rn(make_float2(v[j][k * 4 + 2], v[j][k * 4 + 3]), is2);
      p01 = __fadd2_rn(make_float2(fminf(p01.x, 127.0f), fminf(p01.y, 127.0f)), mg2);
      p23 = __fadd2_rn(make_float2(fminf(p23.x, 127.0f), fminf(p23.y, 127.0f)), mg2);
      w[k] = nz ? pack_low_bytes(__float_as_uint(p01.x), __float_as_uint(p01.y), __float_as_uint(p23.x),
                                 __float_as_uint(p23.y))
                : 0u;
      sum = __dp4a((int)w[k], 0x01010101, sum);
    }
    o.x[j] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  o.sum = sum;
  o.dx = nz ? __fdiv_rn(1.0f, iscale) : 0.0f;
  if (writer) {
    int8_t* dst = (Split<FMT>::xq_out(p) + (int64_t)m * p.ldxq) + (int64_t)b * 256 + vbase;
#pragma unroll
    for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(dst + j * 32) = o.x[j];
    if (cc == 0 && p.xd_out) (Split<FMT>::xd_out(p) + (int64_t)m * p.ldxd)[b] = o.dx;
  }
}

// ------------------------------------------------------------------------------------------------------------------
// Cluster-shared activation prologue: the CTAs of a thread-block cluster split the activation chunks, each quantizes
// its share once (the same load_x_direct arithmetic), keeps it in registers and sends the q8 chunk into every other
// member's shared memory with asynchronous distributed-shared-memory stores (st.async, no multicast loads) that
// complete bytes on the receiver's mbarrier; a thread whose chunk a peer computes waits on that mbarrier (bounded) and
// reads the chunk. No cluster-wide barrier on the critical path: the one that makes the mbarriers visible to the peers
// runs before the dependency wait. Per SM this loads and quantizes 1/cluster of the activations instead of all.
// ------------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_map(uint32_t local_addr, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(local_addr), "r"(rank));
  return a;
}
// asynchronous store into another cluster member's shared memory; its bytes complete on that member's mbarrier rbar
// (both addresses mapped to the member with cluster_map)
__device__ __forceinline__ void st_async_v4(uint32_t addr, uint4 v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(addr),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(rbar)
               : "memory");
}
__device__ __forceinline__ void st_async_v2(uint32_t addr, uint32_t a, uint32_t b, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.b32 [%0], {%1, %2}, [%3];" ::"r"(addr),
               "r"(a), "r"(b), "r"(rbar)
               : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Shared-memory bytes of the chunk slots: [kFields][C] 16-byte q8 pieces, then [C] (sum, scale bits).
template <int FMT>
__host__ __device__ constexpr uint32_t cluster_slot_bytes(int C) {
  return (uint32_t)C * (16u * Fmt<FMT>::kFields + 8u);
}

// Chunks of the activations this cluster member quantizes: warps [rank * per, (rank + 1) * per) (whole warps, for the
// quad shuffles of the q8_K prologue), and the bytes it receives from the other members.
__device__ __forceinline__ int cluster_chunks_per_member(int C, int cs) { return (((C + cs - 1) / cs) + 31) & ~31; }
template <int FMT>
__device__ __forceinline__ uint32_t cluster_recv_bytes(int C, int cs, int rank) {
  const int per = cluster_chunks_per_member(C, cs);
  const int own = max(0, min(per, C - rank * per));
  return (uint32_t)(C - own) * (16u * Fmt<FMT>::kFields + 8u);
}

// xbar: this CTA's mbarrier for the chunks the other members send (initialized with one arrival that expects
// cluster_recv_bytes, made visible to the cluster before any member sends). Returns false if that wait timed out.
template <int FMT>
__device__ __forceinline__ bool cluster_share_x(const GemvParams& p, uint32_t slots, uint32_t xbar, XChunk& xr) {
  const int C = p.C, cs = p.cluster;
  const int per = cluster_chunks_per_member(C, cs);
  const int c = (int)threadIdx.x;
  const int wfirst = c & ~31;
  const int me = (int)cluster_ctarank();
#pragma unroll
  for (int j = 0; j < 4; ++j) xr.x[j] = make_uint4(0u, 0u, 0u, 0u);
  xr.sum = 0;
  xr.dx = 0.f;
  if (wfirst < C && wfirst / per == me) {  // warp-uniform: this member quantizes the warp's chunks
    XChunk o;
    load_x_direct<FMT>(p, c, c < C, o);
    if (c < C) {
      for (int q = 0; q < cs; ++q) {
        if (q == me) continue;
        const uint32_t rbar = cluster_map(xbar, (uint32_t)q);
#pragma unroll
        for (int j = 0; j < Fmt<FMT>::kFields; ++j)
          st_async_v4(cluster_map(slots + (uint32_t)(j * C + c) * 16u, (uint32_t)q), o.x[j], rbar);
        st_async_v2(cluster_map(slots + (uint32_t)Fmt<FMT>::kFields * C * 16u + (uint32_t)c * 8u, (uint32_t)q),
                    (uint32_t)o.sum, __float_as_uint(o.dx), rbar);
      }
      xr = o;
    }
    return true;
  }
  if (c >= C) return true;
  if (!mbar_wait(xbar, 0u, kWaitLimit)) return false;  // every other member's chunks have landed (acquire)
#pragma unroll
  for (int j = 0; j < Fmt<FMT>::kFields; ++j) xr.x[j] = lds_v4(slots + (uint32_t)(j * C + c) * 16u);
  uint32_t a, b;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];"
               : "=r"(a), "=r"(b)
               : "r"(slots + (uint32_t)Fmt<FMT>::kFields * C * 16u + (uint32_t)c * 8u));
  xr.sum = (int)a;
  xr.dx = __uint_as_float(b);
  return true;
}

template <int FMT, int MC, bool XREG>
__device__ __forceinline__ void get_x(const GemvParams& p, const uint8_t* xs, const int* xsum, const float* xscale,
                                      const XChunk (&xr)[MC], int c, bool valid, XChunk (&xc)[MC]) {
  if (XREG) {
#pragma unroll
    for (int m = 0; m < MC; ++m) xc[m] = xr[m];
  } else {
#pragma unroll
    for (int m = 0; m < MC; ++m)
      if (m < p.M) load_xchunk<FMT>(p, xs, xsum, xscale, m, c, valid, xc[m]);
  }
}

template <int FMT, int R, int MC, bool BYTES, bool XREG>
__global__ void __launch_bounds__(kMaxThreads, 1) gemv_reg_kernel(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int C = p.C;
  const int Mx = XREG ? 0 : p.M;  // XREG: activations never touch shared memory
  const int nblk = (int)(p.K / Fmt<FMT>::kBlock);
  uint8_t* xs = smem;                                                    // [Mx][K] permuted int8
  int* xsum = reinterpret_cast<int*>(smem + (size_t)Mx * p.K);            // [Mx][C]
  float* xscale = reinterpret_cast<float*>(xsum + Mx * C);               // [Mx][nblk]
  float* red = xscale + Mx * nblk;                                       // [2][warps][R*MC]

  const int64_t g_begin = (p.groups * blockIdx.x) / gridDim.x;
  const int64_t g_end = (p.groups * (blockIdx.x + 1)) / gridDim.x;

  WeightRegs<R> cur, nxt;
  load_unit<FMT, R>(p, g_begin, 0, g_begin < g_end, cur);
  pdl_wait_then_trigger();
  const int parity = call_parity(p);
  XChunk xr[MC];  // XREG: this thread's only chunk (CPT == 1) of each column, for the whole kernel
  if (XREG) {
#pragma unroll
    for (int m = 0; m < MC; ++m) load_x_direct<FMT>(p, (int)threadIdx.x, (int)threadIdx.x < C && m < p.M, xr[m], m);
  } else
    stage_activations<FMT>(p, xs, xsum, xscale);

  float acc[R * MC];
#pragma unroll
  for (int k = 0; k < R * MC; ++k) acc[k] = 0.f;

  int buf = 0;
  int64_t g = g_begin;
  int i = 0;
  while (g < g_end) {
    int64_t gn = g;
    int in = i + 1;
    if (in == p.CPT) {
      in = 0;
      gn = g + 1;
    }
    load_unit<FMT, R>(p, gn, in, gn < g_end, nxt);

    const int c = (int)threadIdx.x + i * (int)blockDim.x;
    const bool valid = c < C;
    RowScale<FMT> dw[R];
#pragma unroll
    for (int r = 0; r < R; ++r) dw[r].d = f16_bits_to_f32(cur.sc[r]);
    XChunk xc[MC];
    get_x<FMT, MC, XREG>(p, xs, xsum, xscale, xr, c, valid, xc);
    if (p.s)
      compute_chunk<FMT, R, MC, BYTES, true>(p, g, c, valid, cur.w, dw, xc, acc);
    else
      compute_chunk<FMT, R, MC, BYTES, false>(p, g, c, valid, cur.w, dw, xc, acc);
    if (in == 0) {
      reduce_store<R, MC>(p, g, acc, red, buf, parity);
      buf ^= 1;
    }
    cur = nxt;
    g = gn;
    i = in;
  }
  if (p.rx_peers != nullptr) allgather_collect(p, parity);
}

// ------------------------------------------------------------------------------------------------------------------
// Ring path: TMA bulk copies of whole row groups into an S-stage shared-memory ring.
// ------------------------------------------------------------------------------------------------------------------
template <int FMT, int R>
__device__ __forceinline__ void issue_group(const GemvParams& p, int64_t g, uint32_t stage, uint32_t bar,
                                            uint64_t pol) {
  const int nblk = (int)(p.K / Fmt<FMT>::kBlock);
  const uint32_t qrow = (uint32_t)p.C * 16u, srow = (uint32_t)nblk * (uint32_t)Fmt<FMT>::kScaleBytes;
  const int64_t r0 = g * R;
  const int rows = (int)min((int64_t)R, p.N - r0);
  mbar_expect_tx(bar, (uint32_t)rows * (qrow + srow));
  const uint8_t* wq = Split<FMT>::wq(p);
  const int16_t* ws = Split<FMT>::ws(p);
  if (p.dense) {
    bulk_g2s(stage, wq + r0 * p.ldwq, (uint32_t)rows * qrow, bar, pol);
  } else {
    for (int r = 0; r < rows; ++r) bulk_g2s(stage + r * qrow, wq + (r0 + r) * p.ldwq, qrow, bar, pol);
  }
  if (p.ldws == (int64_t)nblk * (Fmt<FMT>::kScaleBytes / 2)) {  // contiguous scale rows: one copy
    bulk_g2s(stage + R * qrow, ws + r0 * p.ldws, (uint32_t)rows * srow, bar, pol);
  } else {
    for (int r = 0; r < rows; ++r) bulk_g2s(stage + R * qrow + r * srow, ws + (r0 + r) * p.ldws, srow, bar, pol);
  }
}

#ifdef B2Q_RING_MAXNREG
#define B2Q_RING_BOUNDS __maxnreg__(B2Q_RING_MAXNREG)
#else
// 16-row groups (one column, one chunk per thread) need more than 128 registers: CTAs of at most 256 threads
#define B2Q_RING_BOUNDS __launch_bounds__(R >= 16 ? 256 : kMaxThreads, 1)
#endif
template <int FMT, int R, int MC, bool XREG>
__global__ void B2Q_RING_BOUNDS gemv_ring_kernel(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_abort;
  __shared__ __align__(8) uint64_t s_xbar;  // clusters: the other members' activation chunks have landed
  const int C = p.C, S = p.stages;
  const int Mx = XREG ? 0 : p.M;  // XREG: activations never touch shared memory
  const int nblk = (int)(p.K / Fmt<FMT>::kBlock);
  const uint32_t qrow = (uint32_t)C * 16u, srow = (uint32_t)nblk * (uint32_t)Fmt<FMT>::kScaleBytes;
  uint8_t* ring = smem;                                                          // [S][stage_bytes]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)S * p.stage_bytes);  // [S]
  uint8_t* xs = reinterpret_cast<uint8_t*>(bars + ((S + 1) & ~1));               // 16-byte aligned
  int* xsum = reinterpret_cast<int*>(xs + (size_t)Mx * p.K);
  float* xscale = reinterpret_cast<float*>(xsum + Mx * C);
  uint8_t* slots = reinterpret_cast<uint8_t*>(xscale + Mx * nblk);  // XREG with clusters: shared chunk slots
  float* red = reinterpret_cast<float*>(slots + ((XREG && p.cluster > 1) ? cluster_slot_bytes<FMT>(C) : 0u));

  const int64_t g_begin = (p.groups * blockIdx.x) / gridDim.x;
  const int64_t g_end = (p.groups * (blockIdx.x + 1)) / gridDim.x;
  const int64_t ngroups = g_end - g_begin;
  const uint32_t ring_addr = smem_addr(ring), bar_addr = smem_addr(bars);
  const uint64_t pol = evict_first_policy();

  const bool share = XREG && MC == 1 && p.cluster > 1;
  const uint32_t xbar = smem_addr(&s_xbar);
  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < S; ++s) mbar_init(bar_addr + 8 * s, 1);
    if (share) {
      mbar_init(xbar, 1);
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(xbar),
                   "r"(cluster_recv_bytes<FMT>(C, p.cluster, (int)cluster_ctarank()))
                   : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // S - 1 groups before the dependency wait; the last stage is filled after the activation prologue. Filling the
    // whole ring up front measured slower (timestamped B200 runs: the extra bulk traffic delays both the preceding
    // grid's completion and this grid's activation loads; gate_up 26.2 vs 25.3 us, down 18.0 vs 17.7 us)
    for (int64_t j = 0; j < min((int64_t)(S - 1), ngroups); ++j)
      issue_group<FMT, R>(p, g_begin + j, ring_addr + (uint32_t)j * p.stage_bytes, bar_addr + 8 * (uint32_t)j, pol);
  }
  // XREG: publish the barrier init and s_abort before the dependency wait (clusters: to every member, before any
  // member sends chunks), so that the activation prologue after it needs no barrier
  if (XREG) {
    if (share)
      cluster_sync_all();
    else
      __syncthreads();
  }
  pdl_wait_then_trigger();
  const int rx_parity = call_parity(p);
  XChunk xr[MC];  // XREG: this thread's only chunk (CPT == 1) of each column, for the whole kernel
  if (XREG) {
    if (share) {
      if (!cluster_share_x<FMT>(p, smem_addr(slots), xbar, xr[0])) {
        s_abort = 1;
        atomicCAS(&g_device_error, 0, kErrTimeout);
      }
    } else {
#pragma unroll
      for (int m = 0; m < MC; ++m)
        load_x_direct<FMT>(p, (int)threadIdx.x, (int)threadIdx.x < C && m < p.M, xr[m], m);
    }
  } else {
    stage_activations<FMT>(p, xs, xsum, xscale);  // ends with __syncthreads (also publishes the barrier init)
  }

  float acc[R * MC];
#pragma unroll
  for (int k = 0; k < R * MC; ++k) acc[k] = 0.f;

  // Stage bookkeeping without divisions: group j sits in stage j % S with mbarrier phase parity (j / S) & 1; the
  // producer refills stage (j - 1) % S with group j + S - 1 (at j = 0 that is the last stage, still unused).
  // The per-group extra work -- issuing the next copy and the cross-warp sum -- rotates over the warps (issuer warp
  // j mod W, summing warp (j + W/2) mod W), so that no warp is the one the others wait for at every barrier.
  const int nwarps = blockDim.x >> 5;
  int iw = 0, fw = nwarps >> 1;
  int buf = 0;
  int s = 0;            // stage of group j
  uint32_t parity = 0;  // phase parity of group j's stage
  int64_t j = 0;
  for (; j < ngroups; ++j) {
    if (threadIdx.x == 32 * iw && j + S - 1 < ngroups) {
      // stage (j-1)%S was released by the previous group's __syncthreads
      const int sn = (s == 0) ? S - 1 : s - 1;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue_group<FMT, R>(p, g_begin + j + S - 1, ring_addr + (uint32_t)sn * p.stage_bytes, bar_addr + 8 * sn, pol);
    }
    if (!mbar_wait(bar_addr + 8 * s, parity, kWaitLimit)) {
      s_abort = 1;
      atomicCAS(&g_device_error, 0, kErrTimeout);
    }
    const uint32_t stage = ring_addr + (uint32_t)s * p.stage_bytes;
    const int64_t g = g_begin + j;
    for (int i = 0; i < (XREG ? 1 : p.CPT); ++i) {
      const int c = (int)threadIdx.x + i * (int)blockDim.x;
      const bool valid = c < C;
      const int blk = c >> Fmt<FMT>::kChunkShift;
      uint4 w[R];
      RowScale<FMT> dw[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (valid) {
          w[r] = lds_v4(stage + r * qrow + (uint32_t)c * 16u);
          dw[r] = row_scale_smem<FMT>(stage + R * qrow + r * srow, c);
        } else {
          w[r] = make_uint4(0u, 0u, 0u, 0u);
          dw[r] = RowScale<FMT>{};
        }
      }
      XChunk xc[MC];
      get_x<FMT, MC, XREG>(p, xs, xsum, xscale, xr, c, valid, xc);
      if (p.s)
        compute_chunk<FMT, R, MC, false, true>(p, g, c, valid, w, dw, xc, acc);
      else
        compute_chunk<FMT, R, MC, false, false>(p, g, c, valid, w, dw, xc, acc);
    }
    reduce_store<R, MC>(p, g, acc, red, buf, rx_parity, fw);
    buf ^= 1;
    if (++s == S) {
      s = 0;
      parity ^= 1u;
    }
    if (++iw == nwarps) iw = 0;
    if (++fw == nwarps) fw = 0;
    if (s_abort) break;  // uniform: read after the reduction's __syncthreads
  }
  if (s_abort) {
    // drain: wait (bounded) for copies that were issued but not consumed (groups j .. j+S-1), then leave
    if (threadIdx.x == 0) {
      for (int64_t jj = j; jj < min(ngroups, j + S); ++jj)
        mbar_wait(bar_addr + 8 * (uint32_t)(jj % S), (uint32_t)((jj / S) & 1), kWaitLimit);
    }
    return;
  }
  if (p.rx_peers != nullptr) allgather_collect(p, rx_parity);
}

// ------------------------------------------------------------------------------------------------------------------
// Warp-rows kernel (one activation column): every warp owns whole weight rows, so a row's sum never leaves its warp.
// ------------------------------------------------------------------------------------------------------------------
// One CTA per SM of W warps. The f32 activations are quantized once per CTA into shared memory (the same permuted
// layout and bytes as the ring path's prologue). Each warp streams its own groups of R rows through its own S-stage
// ring (TMA bulk copies issued by the warp's lane 0, one mbarrier per stage) and takes its next group from a CTA-wide
// counter, so the warps finish together. Lane l computes chunks l, l+32, ... of every row of a group; the group's R
// sums are reduced inside the warp once per group, so the per-group cost is spread over all of a lane's chunks and the
// loop has no CTA-wide barrier. The whole ring (W x S groups) is requested before the activation prologue.
// Shared memory: [W][S] stages, [W][S] mbarriers, activations (K bytes), chunk sums (C ints), block scales.
template <int FMT, int R>
__global__ void __launch_bounds__(kMaxThreads, 1) gemv_warp_kernel(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_next;                                    // next unassigned group of this CTA
  __shared__ int s_abort;
  __shared__ int s_group[kMaxThreads / 32][kMaxStages];    // CTA-local group held by each warp's stage, -1: none
  const int C = p.C, S = p.stages, W = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nblk = (int)(p.K / Fmt<FMT>::kBlock);
  const uint32_t qrow = (uint32_t)C * 16u, srow = (uint32_t)nblk * (uint32_t)Fmt<FMT>::kScaleBytes;
  uint8_t* ring = smem;                                                                   // [W][S][stage_bytes]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)W * S * p.stage_bytes);    // [W][S]
  uint8_t* xs = reinterpret_cast<uint8_t*>(bars + ((W * S + 1) & ~1));                   // 16-byte aligned
  int* xsum = reinterpret_cast<int*>(xs + (size_t)p.K);
  float* xscale = reinterpret_cast<float*>(xsum + C);

  const int64_t g_begin = (p.groups * blockIdx.x) / gridDim.x;
  const int n = (int)((p.groups * (blockIdx.x + 1)) / gridDim.x - g_begin);
  const uint32_t my_ring = smem_addr(ring) + (uint32_t)(warp * S) * p.stage_bytes;
  const uint32_t my_bars = smem_addr(bars) + (uint32_t)(warp * S) * 8u;
  const uint64_t pol = evict_first_policy();

  // Initial fills (weights only, so before the dependency wait): warp w's stage k gets group k*W + w.
  if (lane == 0) {
    for (int k = 0; k < S; ++k) mbar_init(my_bars + 8 * k, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int k = 0; k < S; ++k) {
      const int gl = k * W + warp;
      if (gl < n) issue_group<FMT, R>(p, g_begin + gl, my_ring + (uint32_t)k * p.stage_bytes, my_bars + 8 * k, pol);
      s_group[warp][k] = gl < n ? gl : -1;
    }
  }
  if (threadIdx.x == 0) {
    s_next = S * W;
    s_abort = 0;
  }
  pdl_wait_then_trigger();
  stage_activations<FMT>(p, xs, xsum, xscale);  // ends with __syncthreads (publishes the inits above)

  int s = 0;
  uint32_t parity = 0;
  while (true) {
    const int gl = *reinterpret_cast<volatile int*>(&s_group[warp][s]);
    if (gl < 0) break;  // warp-uniform: groups are handed out in increasing order, so the rest are empty too
    const bool ok = __all_sync(0xffffffffu, mbar_wait(my_bars + 8 * s, parity, kWaitLimit));
    if (!ok || *reinterpret_cast<volatile int*>(&s_abort)) {
      if (lane == 0) {
        *reinterpret_cast<volatile int*>(&s_abort) = 1;
        if (!ok) atomicCAS(&g_device_error, 0, kErrTimeout);
        // drain (bounded): this warp's copies still in flight, in ring order from stage s
        for (int k = 0; k < S; ++k) {
          const int st = (s + k) % S;
          if (*reinterpret_cast<volatile int*>(&s_group[warp][st]) >= 0)
            mbar_wait(my_bars + 8 * st, parity ^ (st < s ? 1u : 0u), kWaitLimit);
        }
      }
      break;
    }
    const uint32_t stage = my_ring + (uint32_t)s * p.stage_bytes;
    const int64_t g = g_begin + gl;
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    for (int i = 0; i < p.CPT; ++i) {
      const int c = lane + 32 * i;
      const bool valid = c < C;
      const int blk = c >> Fmt<FMT>::kChunkShift;
      uint4 w[R];
      RowScale<FMT> dw[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (valid) {
          w[r] = lds_v4(stage + r * qrow + (uint32_t)c * 16u);
          dw[r] = row_scale_smem<FMT>(stage + R * qrow + r * srow, c);
        } else {
          w[r] = make_uint4(0u, 0u, 0u, 0u);
          dw[r] = RowScale<FMT>{};
        }
      }
      XChunk xc[1];
      load_xchunk<FMT>(p, xs, xsum, xscale, 0, c, valid, xc[0]);
      if (p.s)
        compute_chunk<FMT, R, 1, false, true>(p, g, c, valid, w, dw, xc, acc);
      else
        compute_chunk<FMT, R, 1, false, false>(p, g, c, valid, w, dw, xc, acc);
    }
    const float v = warp_sum_scatter<R>(acc, lane);
    if ((lane & (32 / R - 1)) == 0) {
      const int64_t row = g * R + lane / (32 / R);
      if (row < p.N) p.y[p.row0 + row] = v;
    }
    __syncwarp();
    if (lane == 0) {  // every lane's reads of this stage are done: refill it with the CTA's next group
      const int nx = atomicAdd(&s_next, 1);
      if (nx < n && !*reinterpret_cast<volatile int*>(&s_abort)) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue_group<FMT, R>(p, g_begin + nx, stage, my_bars + 8 * s, pol);
        s_group[warp][s] = nx;
      } else {
        s_group[warp][s] = -1;
      }
    }
    __syncwarp();
    if (++s == S) {
      s = 0;
      parity ^= 1u;
    }
  }
}

using KernelFn = void (*)(const GemvParams);

// Kernel selection, one per translation unit (instantiations live in gemv_reg.cu / gemv_ring.cu).
KernelFn reg_kernel_for(int fmt, bool bytes, int R, int MC, bool xreg);
KernelFn ring_kernel_for(int fmt, int R, int MC, bool xreg);
KernelFn warp_kernel_for(int fmt, int R);

}  // namespace b2q
