// Batched quantized GEMM on the 5th-generation tensor cores (tcgen05, kind::i8) for many activation columns.
//
// The GEMV kernels re-read the weights once per group of 4 columns; for M >= 8 columns (prefill, speculative or
// batched decode) this kernel reads them once and lets the tensor cores do the integer dot products. Same results as
// the GEMVs: every block dot is the exact int32 sum (read from tensor memory per block), Y adds the per-block f32
// products in the reference's multiply order (Q4_0: f32(s) * dw * dx, TQ2_0: dx * dw * f32(s); kernels.py:93, 141).
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
#include "gemv_kernels.cuh"

namespace b2q {

namespace tc {

__device__ __forceinline__ int core_off(int r, int kb) {  // byte offset of (row r, k-byte kb) in a K-major tile
  return (r & 7) * 16 + (kb >> 4) * 128 + (r >> 3) * 256 + (kb & 15);
}
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {  // no swizzle; LBO 128 B (next 16 k-bytes), SBO 256 B
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) |
         ((uint64_t)1 << 46);
}
// kind::i8 instruction descriptor: s32 accumulator, A unsigned 8-bit, B signed 8-bit, both K-major, M = 128, N = nt
__device__ __forceinline__ uint32_t instr_desc(int nt) {
  return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(nt >> 3) << 17) | (8u << 24);
}
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                 "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

}  // namespace tc

// Epilogue of block b (accumulator buf): this row's exact int32 dots -> offset -> scaled f32 sums; S dump if STORE.
template <int FMT, int NT, bool STORE>
__device__ __forceinline__ void gemm_tc_finish(const GemvParams& p, uint32_t tmem_row, uint64_t* full, int b,
                                               const int (&xsum)[3][NT], const float (&xdx)[3][NT], int slot,
                                               float dw, float (&acc)[NT], bool& timed_out, int64_t row,
                                               int64_t col0, int ncols, int nblk, bool row_ok) {
  const int buf = b & 1;
  if (!mbar_wait(smem_addr(&full[buf]), (uint32_t)((b >> 1) & 1), kWaitLimit)) timed_out = true;
  tc::fence_after();
#pragma unroll
  for (int c0 = 0; c0 < NT; c0 += 16) {
    uint32_t v[16];
    tc::tmem_ld16(tmem_row + (uint32_t)(buf * NT + c0), v);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int c = c0 + j;
      const int s = (int)v[j] - (FMT == 0 ? 8 : 1) * xsum[slot][c];
      if (FMT == 0)
        acc[c] = __fmaf_rn(__fmul_rn((float)s, dw), xdx[slot][c], acc[c]);
      else
        acc[c] = __fmaf_rn(__fmul_rn(xdx[slot][c], dw), (float)s, acc[c]);
      if (STORE && row_ok && c < ncols) p.s[((col0 + c) * p.N + row) * nblk + b] = s;
    }
  }
  tc::fence_before();
}

// FMT 0: Q4_0 (1 MMA per block), FMT 1: TQ2_0 (8 MMAs per block). NT activation columns per CTA.
template <int FMT, int NT, bool STORE>
__global__ void __launch_bounds__(128) gemm_tc_kernel(const GemvParams p) {
  constexpr int KS = FMT == 0 ? 1 : 8;      // MMAs (32-value k-steps) per weight block
  constexpr int ATILE = 128 * 32;           // A bytes per k-step
  constexpr int BTILE = NT * 32;            // B bytes per k-step
  constexpr int NCOLS = 2 * NT < 32 ? 32 : 2 * NT;  // two accumulators
  extern __shared__ __align__(128) uint8_t tc_smem[];
  uint8_t* sA = tc_smem;                                             // [2][KS][ATILE]
  int8_t* sB = reinterpret_cast<int8_t*>(tc_smem + 2 * KS * ATILE);  // [2][KS][BTILE]
  __shared__ __align__(8) uint64_t full[2];
  // block sums and scales of the columns: three slots (block b in slot b % 3), because a thread may still read block
  // b - 1's while another already stages block b + 1's (operands and accumulators are only reused after waits)
  __shared__ int s_xsum[3][NT];
  __shared__ float s_dx[3][NT];
  __shared__ uint32_t s_tmem;

  const int t = threadIdx.x, warp = t >> 5;
  const int64_t row0 = (int64_t)blockIdx.x * 128, col0 = (int64_t)blockIdx.y * NT;
  const int64_t row = row0 + t;
  const bool row_ok = row < p.N;
  const int ncols = (int)min((int64_t)NT, (int64_t)p.M - col0);
  const int nblk = (int)(p.K / Fmt<FMT>::kBlock);
  const uint8_t* wrow = p.wq + (row_ok ? row : 0) * p.ldwq;
  const int16_t* srow = p.ws + (row_ok ? row : 0) * p.ldws;
  const uint32_t idesc = tc::instr_desc(NT);

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
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = s_tmem;
  const uint32_t lane_base = (uint32_t)(32 * warp) << 16;

  float acc[NT];
#pragma unroll
  for (int c = 0; c < NT; ++c) acc[c] = 0.f;
  bool timed_out = false;

  int slot = 0, prev_slot = 2;  // b % 3, (b - 1) % 3
  for (int b = 0; b < nblk; ++b) {
    const int buf = b & 1;
    uint8_t* a = sA + buf * KS * ATILE;
    int8_t* bt = sB + buf * KS * BTILE;
    // A: this row's block, unpacked to unsigned bytes in natural value order (k-step s = values 32s .. 32s+31)
    if (FMT == 0) {
      uint4 w = make_uint4(0u, 0u, 0u, 0u);
      if (row_ok) w = *reinterpret_cast<const uint4*>(wrow + (int64_t)b * 16);
      const uint4 lo = make_uint4(w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, w.z & 0x0F0F0F0Fu, w.w & 0x0F0F0F0Fu);
      const uint4 hi = make_uint4((w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu, (w.z >> 4) & 0x0F0F0F0Fu,
                                  (w.w >> 4) & 0x0F0F0F0Fu);
      *reinterpret_cast<uint4*>(a + tc::core_off(t, 0)) = lo;   // values 0..15: low nibbles of bytes 0..15
      *reinterpret_cast<uint4*>(a + tc::core_off(t, 16)) = hi;  // values 16..31: high nibbles
    } else {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint4 q[2];
#pragma unroll
        for (int u = 0; u < 2; ++u)
          q[u] = row_ok ? *reinterpret_cast<const uint4*>(wrow + (int64_t)b * 64 + h * 32 + u * 16)
                        : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {  // k-step 4h + j: field j of bytes h*32 .. h*32+31 = values h*128 + 32j + t
          const int sh = 2 * j;
          uint8_t* as = a + (4 * h + j) * ATILE;
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const uint4 f = make_uint4((q[u].x >> sh) & 0x03030303u, (q[u].y >> sh) & 0x03030303u,
                                       (q[u].z >> sh) & 0x03030303u, (q[u].w >> sh) & 0x03030303u);
            *reinterpret_cast<uint4*>(as + tc::core_off(t, 16 * u)) = f;
          }
        }
      }
    }
    // B: the block's activations of this CTA's columns (zero for columns past M), the column block sums and scales
    {
      constexpr int PIECES = KS * NT * 2;  // 16-byte pieces: (k-step, column, half)
      for (int i = t; i < PIECES; i += 128) {
        const int s = i / (NT * 2), rem = i - s * NT * 2, c = rem >> 1, half = rem & 1;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (c < ncols)
          v = *reinterpret_cast<const uint4*>(p.xq + (col0 + c) * p.ldxq + (int64_t)b * Fmt<FMT>::kBlock + s * 32 +
                                              half * 16);
        *reinterpret_cast<uint4*>(bt + s * BTILE + tc::core_off(c, 16 * half)) = v;
      }
      if (t < NT) {
        int sum = 0;
        float dx = 0.f;
        if (t < ncols) {
          const int8_t* xc = p.xq + (col0 + t) * p.ldxq + (int64_t)b * Fmt<FMT>::kBlock;
#pragma unroll
          for (int u = 0; u < Fmt<FMT>::kBlock / 16; ++u) {
            const uint4 v = *reinterpret_cast<const uint4*>(xc + u * 16);
            sum += bytesum(v.x) + bytesum(v.y) + bytesum(v.z) + bytesum(v.w);
          }
          dx = p.xd[(col0 + t) * p.ldxd + b];
        }
        s_xsum[slot][t] = sum;
        s_dx[slot][t] = dx;
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic stores -> tensor-core reads
    tc::fence_before();
    __syncthreads();  // operands of block b complete; every thread finished block b - 2's epilogue
    tc::fence_after();
    if (t == 0) {
#pragma unroll
      for (int s = 0; s < KS; ++s)
        tc::mma_i8(tmem + (uint32_t)(buf * NT), tc::smem_desc(smem_addr(a + s * ATILE)),
                   tc::smem_desc(smem_addr(bt + s * BTILE)), idesc, s > 0 ? 1u : 0u);
      tc::mma_commit(smem_addr(&full[buf]));
    }
    if (b > 0)
      gemm_tc_finish<FMT, NT, STORE>(p, tmem + lane_base, full, b - 1, s_xsum, s_dx, prev_slot,
                                     f16_bits_to_f32((uint16_t)srow[b - 1]), acc, timed_out, row, col0, ncols, nblk,
                                     row_ok);
    prev_slot = slot;
    slot = slot == 2 ? 0 : slot + 1;
  }
  if (nblk > 0)
    gemm_tc_finish<FMT, NT, STORE>(p, tmem + lane_base, full, nblk - 1, s_xsum, s_dx, prev_slot,
                                   f16_bits_to_f32((uint16_t)srow[nblk - 1]), acc, timed_out, row, col0, ncols, nblk,
                                   row_ok);

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
  constexpr int KS = FMT == 0 ? 1 : 8;
  return (size_t)2 * KS * (128 * 32 + NT * 32);
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
  return after_launch(fmt == 0 ? "gemm_tc_q4_0" : "gemm_tc_tq2_0");
}

}  // namespace b2q
