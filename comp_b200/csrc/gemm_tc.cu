// Batched quantized GEMM on the 5th-generation tensor cores (tcgen05, kind::i8) for many activation columns.
//
// The GEMV kernels re-read the weights once per group of 4 columns; for M >= 8 columns (prefill, speculative or
// batched decode) this kernel reads them once and lets the tensor cores do the integer dot products. Same results as
// the GEMVs: every block dot is the exact int32 sum (read from tensor memory per block), Y adds the per-block f32
// products in the reference's multiply order (Q4_0: f32(s) * dw * dx, TQ2_0: dx * dw * f32(s); kernels.py:93, 141).
//
// Q8_0 weights (format 2, an extension beyond the reference) take the same path with signed A and no offset.
//
// One CTA of 128 threads computes 128 weight rows x NT activation columns (NT = 16 .. 128, grid.y covers more).
// Thread t owns weight row t = tensor-memory lane t. Per weight block (Q4_0: 32 values, one MMA with K = 32; TQ2_0:
// 256 values, eight MMAs accumulated):
//   1. every thread loads its row's packed block, unpacks the 4-bit (Q4_0) or 2-bit (TQ2_0) fields to unsigned bytes
//      and stores them as the A operand (128 x 32 bytes per MMA, K-major, 8-row x 16-byte core matrices, no swizzle);
//      the threads stage the block's activations (NT x 32 bytes per MMA) as the B operand, and thread c < NT the
//      column's block sum (the weights' offset -8 / -1 is applied as -8 * sum(x) / -sum(x));
//   2. one thread issues the block's MMAs into one of two tensor-memory accumulators (NT int32 columns each) and
//      commits them to that accumulator's mbarrier;
//   3. meanwhile every thread finishes the previous block: waits for its accumulator, reads its row's NT int32 dots
//      (tcgen05.ld), subtracts the offset and adds the scaled products into NT f32 registers.
// Operands and accumulators are double-buffered, so the MMA of block b overlaps the epilogue of block b - 1. Every
// wait is bounded; on a timeout the kernel sets the device error word and still frees its tensor memory.
#include "tc_device.cuh"

namespace b2q {


// Epilogue of block b (accumulator buf): this row's exact int32 dots -> offset -> scaled f32 sums; S dump if STORE.
// Epilogue of block group i (accumulator buf = i & 1, block i*G + j in region buf * G + j): this row's exact int32
// dots -> offset -> scaled f32 sums; S dump if STORE. Per column, koff = 0x4B400000 - off * sum(x) turns the dot into
// the f32 bit pattern of 2^23 + 2^22 + s (exact for |s| < 2^22), so f32(s) is one integer add and one exact subtract;
// the f32 products then run two columns per instruction (packed FP32x2), in the reference's multiply order.
template <int FMT, int NT, int G, bool STORE>
__device__ __forceinline__ void gemm_tc_finish(const GemvParams& p, uint32_t tmem_row, uint64_t* full, int i, int nb,
                                               const int (&koff)[3][G][NT], const float (&xdx)[3][G][NT], int slot,
                                               const uint16_t (&sc)[G], float (&acc)[NT], bool& timed_out,
                                               int64_t row, int64_t col0, int ncols, int nblk, bool row_ok) {
  constexpr float kMagic = 12582912.0f;  // 2^23 + 2^22
  const int buf = i & 1;
  if (!mbar_wait(smem_addr(&full[buf]), (uint32_t)((i >> 1) & 1), kWaitLimit)) timed_out = true;
  tc::fence_after();
#pragma unroll
  for (int j = 0; j < G; ++j) {
    if (j < nb) {
      const float dw = f16_bits_to_f32(sc[j]);
      const float2 dw2 = make_float2(dw, dw);
#pragma unroll
      for (int c0 = 0; c0 < NT; c0 += 16) {
        uint32_t v[16];
        tc::tmem_ld16(tmem_row + (uint32_t)((buf * G + j) * NT + c0), v);
#pragma unroll
        for (int q = 0; q < 16; q += 2) {
          const int c = c0 + q;
          const float2 f = __fadd2_rn(make_float2(__int_as_float((int)v[q] + koff[slot][j][c]),
                                                  __int_as_float((int)v[q + 1] + koff[slot][j][c + 1])),
                                      make_float2(-kMagic, -kMagic));  // exact f32(s) of both columns
          const float2 dx2 = make_float2(xdx[slot][j][c], xdx[slot][j][c + 1]);
          float2 a2 = make_float2(acc[c], acc[c + 1]);
          if (FMT != 1)
            a2 = __ffma2_rn(__fmul2_rn(f, dw2), dx2, a2);  // f32(s) * dw * dx
          else
            a2 = __ffma2_rn(__fmul2_rn(dx2, dw2), f, a2);  // dx * dw * f32(s)
          acc[c] = a2.x;
          acc[c + 1] = a2.y;
          if (STORE && row_ok) {
            const int64_t base = ((col0 + c) * p.N + row) * nblk + i * G + j;
            if (c < ncols) p.s[base] = (int)v[q] + koff[slot][j][c] - 0x4B400000;
            if (c + 1 < ncols) p.s[base + p.N * nblk] = (int)v[q + 1] + koff[slot][j][c + 1] - 0x4B400000;
          }
        }
      }
    }
  }
  tc::fence_before();
}


// Shape of the pipeline per format and column tile: G weight blocks per iteration (one barrier, one commit and one
// accumulator wait per group), groups fetched ahead, and the shared-memory layout.
template <int FMT, int NT>
struct TcCfg {
  static constexpr int KS = FMT == 1 ? 8 : 1;                  // MMAs (32-value k-steps) per weight block
  static constexpr int QU = FMT == 0 ? 1 : FMT == 1 ? 4 : 2;  // 16-byte units of a row's packed block
  // G = 1: measured on B200, larger groups (more shared memory, fewer resident CTAs) were slower for Q4_0
  static constexpr int G = 1;
  static constexpr int P = FMT == 0 ? 8 : FMT == 2 ? 6 : (NT <= 64 ? 4 : 2);
  static constexpr int ATILE = 128 * 32, BTILE = NT * 32;
  static constexpr size_t RAW = (size_t)P * G * QU * 128 * 16;    // [P][G][QU][128 threads] 16-byte units
  static constexpr size_t ATILES = (size_t)2 * G * KS * ATILE;     // [2][G][KS] unpacked weight tiles
  static constexpr size_t BRING = (size_t)P * G * KS * BTILE;      // [P][G][KS] activation tiles
  static constexpr size_t SMEM = RAW + ATILES + BRING;
  static constexpr int NCOLS = 2 * G * NT < 32 ? 32 : 2 * G * NT;  // two accumulator sets of G x NT columns
};

// FMT 0: Q4_0 (1 MMA per block), FMT 1: TQ2_0 (8 MMAs per block). NT activation columns per CTA.
template <int FMT, int NT, bool STORE>
__global__ void __launch_bounds__(128) gemm_tc_kernel(const GemvParams p) {
  using Cfg = TcCfg<FMT, NT>;
  constexpr int KS = Cfg::KS, QU = Cfg::QU, G = Cfg::G, P = Cfg::P, ATILE = Cfg::ATILE, BTILE = Cfg::BTILE;
  constexpr int NCOLS = Cfg::NCOLS;
  extern __shared__ __align__(128) uint8_t tc_smem[];
  uint8_t* raw = tc_smem;                                    // own-row packed blocks, fetched P - 1 groups ahead
  uint8_t* sA = tc_smem + Cfg::RAW;                          // [2][G][KS][ATILE]
  int8_t* sB = reinterpret_cast<int8_t*>(sA + Cfg::ATILES);  // [P][G][KS][BTILE]
  __shared__ __align__(8) uint64_t full[2];
  // per column and block: 0x4B400000 - offset * sum(x) and the scale, in three slots (group i in slot i % 3), because
  // a thread may still read group i - 1's while another already stages group i + 1's (tiles and accumulators are only
  // reused after waits)
  __shared__ int s_koff[3][G][NT];
  __shared__ float s_dx[3][G][NT];
  __shared__ uint32_t s_tmem;

  const int t = threadIdx.x, warp = t >> 5;
  const int64_t row0 = (int64_t)blockIdx.x * 128, col0 = (int64_t)blockIdx.y * NT;
  const int64_t row = row0 + t;
  const bool row_ok = row < p.N;
  const int ncols = (int)min((int64_t)NT, (int64_t)p.M - col0);
  const int nblk = (int)(p.K / Fmt<FMT>::kBlock);
  const int ngrp = (nblk + G - 1) / G;
  const uint8_t* wrow = p.wq + (row_ok ? row : 0) * p.ldwq;
  const int16_t* srow = p.ws + (row_ok ? row : 0) * p.ldws;
  const uint32_t idesc = tc::instr_desc(NT, FMT == 2);  // Q8_0 weights are signed
  const uint32_t raw_base = smem_addr(raw), b_base = smem_addr(sB);

  // issue the copies of group i (this thread's row's packed blocks; its share of the activation tiles); one group
  auto fetch = [&](int i) {
    if (i < ngrp) {
      const int rs = i % P;
#pragma unroll
      for (int j = 0; j < G; ++j) {
        const int b = i * G + j;
#pragma unroll
        for (int u = 0; u < QU; ++u)
          cp_async16(raw_base + (uint32_t)((((rs * G + j) * QU + u) * 128 + t) * 16),
                     wrow + (int64_t)min(b, nblk - 1) * (QU * 16) + u * 16, row_ok && b < nblk);
      }
      constexpr int PIECES = G * KS * NT * 2;  // (block, k-step, column, half) 16-byte pieces
      for (int q = t; q < PIECES; q += 128) {
        const int js = q / (NT * 2), rem = q - js * NT * 2, c = rem >> 1, half = rem & 1;
        const int j = js / KS, s = js - j * KS, b = i * G + j;
        const bool ok = c < ncols && b < nblk;
        const int8_t* src =
            p.xq + (ok ? (col0 + c) * p.ldxq + (int64_t)b * Fmt<FMT>::kBlock + s * 32 + half * 16 : 0);
        cp_async16(b_base + (uint32_t)(((rs * G + j) * KS + s) * BTILE + tc::core_off(c, 16 * half)), src, ok);
      }
    }
    cp_async_commit();
  };

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                 "r"(NCOLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (t == 0) {
    mbar_init(smem_addr(&full[0]), 1);
    mbar_init(smem_addr(&full[1]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  pdl_wait_then_trigger();
#pragma unroll
  for (int i = 0; i < P - 1; ++i) fetch(i);
  // per-block scales of this row and column scales, one group ahead in registers
  uint16_t sc_pending[G], sc_prev[G], sc_fin[G];
  float dx_next[G];
#pragma unroll
  for (int j = 0; j < G; ++j) {
    sc_pending[j] = (row_ok && j < nblk) ? (uint16_t)srow[j] : (uint16_t)0;
    sc_prev[j] = 0;
    dx_next[j] = (t < ncols && j < nblk) ? p.xd[(col0 + t) * p.ldxd + j] : 0.f;
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = s_tmem;
  const uint32_t lane_base = (uint32_t)(32 * warp) << 16;

  float acc[NT];
#pragma unroll
  for (int c = 0; c < NT; ++c) acc[c] = 0.f;
  bool timed_out = false;

  int slot = 0, prev_slot = 2;  // i % 3, (i - 1) % 3
  for (int i = 0; i < ngrp; ++i) {
    const int buf = i & 1, rs = i % P;
    const int nb = min(G, nblk - i * G);
    uint8_t* a = sA + buf * G * KS * ATILE;
    cp_async_wait<P - 2>();  // this thread's copies of group i have landed
    // A: this row's blocks, unpacked to unsigned bytes in natural value order (k-step s = values 32s .. 32s+31)
#pragma unroll
    for (int j = 0; j < G; ++j) {
      uint8_t* aj = a + j * KS * ATILE;
      const uint32_t rj = raw_base + (uint32_t)((rs * G + j) * QU * 128 * 16);
      if (FMT == 2) {  // Q8_0: the 32 int8 values as they are
        *reinterpret_cast<uint4*>(aj + tc::core_off(t, 0)) = lds_v4(rj + (uint32_t)(t * 16));
        *reinterpret_cast<uint4*>(aj + tc::core_off(t, 16)) = lds_v4(rj + (uint32_t)((128 + t) * 16));
      } else if (FMT == 0) {
        const uint4 w = lds_v4(rj + (uint32_t)(t * 16));
        const uint4 lo = make_uint4(w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, w.z & 0x0F0F0F0Fu, w.w & 0x0F0F0F0Fu);
        const uint4 hi = make_uint4((w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu, (w.z >> 4) & 0x0F0F0F0Fu,
                                    (w.w >> 4) & 0x0F0F0F0Fu);
        *reinterpret_cast<uint4*>(aj + tc::core_off(t, 0)) = lo;   // values 0..15: low nibbles of bytes 0..15
        *reinterpret_cast<uint4*>(aj + tc::core_off(t, 16)) = hi;  // values 16..31: high nibbles
      } else {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint4 q[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) q[u] = lds_v4(rj + (uint32_t)(((2 * h + u) * 128 + t) * 16));
#pragma unroll
          for (int f = 0; f < 4; ++f) {  // k-step 4h + f: field f of bytes h*32 .. h*32+31 = values h*128 + 32f + t
            const int sh = 2 * f;
            uint8_t* as = aj + (4 * h + f) * ATILE;
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const uint4 v = make_uint4((q[u].x >> sh) & 0x03030303u, (q[u].y >> sh) & 0x03030303u,
                                         (q[u].z >> sh) & 0x03030303u, (q[u].w >> sh) & 0x03030303u);
              *reinterpret_cast<uint4*>(as + tc::core_off(t, 16 * u)) = v;
            }
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < G; ++j) {
      if (t < NT) {  // this group's column scales (fetched one group ahead) and the next group's fetch
        s_dx[slot][j][t] = dx_next[j];
        const int bn = (i + 1) * G + j;
        dx_next[j] = (t < ncols && bn < nblk) ? p.xd[(col0 + t) * p.ldxd + bn] : 0.f;
      }
      sc_fin[j] = sc_prev[j];      // scales of group i - 1 (its epilogue below)
      sc_prev[j] = sc_pending[j];  // scales of group i (its epilogue in the next iteration)
      const int bn = (i + 1) * G + j;
      sc_pending[j] = (row_ok && bn < nblk) ? (uint16_t)srow[bn] : (uint16_t)0;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic stores -> tensor-core reads
    tc::fence_before();
    __syncthreads();  // group i's operands complete (all threads' copies); group i - 2's epilogue done everywhere
    tc::fence_after();
    const int8_t* bt = sB + rs * G * KS * BTILE;
    if (t == 0) {
#pragma unroll
      for (int j = 0; j < G; ++j)
        if (j < nb)
#pragma unroll
          for (int s = 0; s < KS; ++s)
            tc::mma_i8(tmem + (uint32_t)((buf * G + j) * NT), tc::smem_desc(smem_addr(a + (j * KS + s) * ATILE)),
                       tc::smem_desc(smem_addr(bt + (j * KS + s) * BTILE)), idesc, s > 0 ? 1u : 0u);
      tc::mma_commit(smem_addr(&full[buf]));
    }
    if (t < NT && Fmt<FMT>::kOffset == 0) {
#pragma unroll
      for (int j = 0; j < G; ++j) s_koff[slot][j][t] = 0x4B400000;  // no offset to fold in
    } else if (t < NT) {  // column block sums from the staged tiles
#pragma unroll
      for (int j = 0; j < G; ++j) {
        int sum = 0;
#pragma unroll
        for (int s = 0; s < KS; ++s)
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const uint4 v = lds_v4(smem_addr(bt + (j * KS + s) * BTILE + tc::core_off(t, 16 * half)));
            sum += bytesum(v.x) + bytesum(v.y) + bytesum(v.z) + bytesum(v.w);
          }
        s_koff[slot][j][t] = 0x4B400000 - Fmt<FMT>::kOffset * sum;
      }
    }
    if (i > 0)
      gemm_tc_finish<FMT, NT, G, STORE>(p, tmem + lane_base, full, i - 1, G, s_koff, s_dx, prev_slot, sc_fin, acc,
                                        timed_out, row, col0, ncols, nblk, row_ok);
    fetch(i + P - 1);  // into the ring slot of group i - 1, whose MMAs this thread has seen complete
    prev_slot = slot;
    slot = slot == 2 ? 0 : slot + 1;
  }
  // the last group's column offsets were written after its barrier: one more barrier before every thread reads them
  __syncthreads();
  if (ngrp > 0)
    gemm_tc_finish<FMT, NT, G, STORE>(p, tmem + lane_base, full, ngrp - 1, nblk - (ngrp - 1) * G, s_koff, s_dx,
                                      prev_slot, sc_prev, acc, timed_out, row, col0, ncols, nblk, row_ok);
  cp_async_wait<0>();

  if (row_ok)
#pragma unroll
    for (int c = 0; c < NT; ++c)
      if (c < ncols) p.y[(col0 + c) * p.ldy + p.row0 + row] = acc[c];
  if (timed_out) atomicCAS(&g_device_error, 0, kErrTimeout);
  tc::fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(NCOLS));
}

template <int FMT, int NT>
static size_t gemm_tc_smem() {
  return TcCfg<FMT, NT>::SMEM;
}

// Launches the tensor-core GEMM for M >= 8 columns (pre-quantized activations). Returns B2Q_OK, or a negative code.
int launch_gemm_tc(const GemvParams& base, int fmt, cudaStream_t stream, bool pdl) {
  const int64_t M = base.M;
  const int NT = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
  KernelFn fn = nullptr;
  size_t smem = 0;
  const bool store = base.s != nullptr;
#define B2Q_TC_CASE(F, T)                                                   \
  if (fmt == F && NT == T) {                                                \
    fn = store ? gemm_tc_kernel<F, T, true> : gemm_tc_kernel<F, T, false>;  \
    smem = gemm_tc_smem<F, T>();                                            \
  }
  B2Q_TC_CASE(0, 16) B2Q_TC_CASE(0, 32) B2Q_TC_CASE(0, 64) B2Q_TC_CASE(0, 128)
  B2Q_TC_CASE(1, 16) B2Q_TC_CASE(1, 32) B2Q_TC_CASE(1, 64) B2Q_TC_CASE(1, 128)
  B2Q_TC_CASE(2, 16) B2Q_TC_CASE(2, 32) B2Q_TC_CASE(2, 64) B2Q_TC_CASE(2, 128)
#undef B2Q_TC_CASE
  if (!fn) return fail(B2Q_EINVAL, "gemm_tc: no kernel for fmt %d", fmt);
  cudaError_t e = cudaFuncSetAttribute((const void*)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return fail(B2Q_ECUDA, "gemm_tc: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((base.N + 127) / 128), (unsigned)((M + NT - 1) / NT));
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, fn, base);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(B2Q_ECUDA, "gemm_tc: launch failed: %s", cudaGetErrorString(e));
  }
  return after_launch(fmt == 0 ? "gemm_tc_q4_0" : fmt == 1 ? "gemm_tc_tq2_0" : "gemm_tc_q8_0");
}

}  // namespace b2q
