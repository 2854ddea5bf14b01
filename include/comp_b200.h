/*
 * comp_b200.h -- C ABI of the B200-native quantized decode path.
 *
 * Four operations on KURN's `split` layout, each a drop-in for one COMP (komp) Triton kernel:
 *
 *   quant_q8_0   f32 activations [M][K] -> int8 XQ [M][K] + f32 XD [M][K/32]   (ggml quantize_row_q8_0_ref)
 *   quant_q8_K   f32 activations [M][K] -> int8 XQ [M][K] + f32 XD [M][K/256]  (ggml quantize_row_q8_K_ref)
 *   gemv_q4_0    Q4_0 weights (WQ u8 [N][K/2], WS f16 bits [N][K/32]) x q8_0 activations -> Y f32 [M][N]
 *   gemv_tq2_0   TQ2_0 weights (WQ u8 [N][K/4], WS f16 bits [N][K/256]) x q8_K activations -> Y f32 [M][N]
 *
 * Conventions shared by every entry point:
 *   - All data pointers are DEVICE pointers of the current CUDA device, except the host buffers of the pinned
 *     entry points (b2q_quant_gemv_pinned, b2q_stage_pinned, b2q_host_device_pointer), which must be page-locked
 *     host memory mapped for that device and are checked before any launch; the library never allocates or frees
 *     device memory (the caller owns every buffer).
 *   - Sizes and strides are int64 element counts (bytes for u8/i8 planes).
 *   - Work is enqueued on `stream` (NULL = legacy default stream) and is asynchronous.
 *   - Return 0 on success, a negative B2Q_E* code otherwise; b2q_last_error() gives the message for the calling
 *     thread. Nothing aborts the process.
 *   - Alignment: x, xq and wq must be 16-byte aligned, with ldx % 4 == 0 and ldwq % 16 == 0 (the layouts the
 *     reference's typed signatures assume: 16-byte aligned pointers, K % 32 == 0).
 *
 * The matching COMP (reference) interfaces are cited per entry point as path:line inside the komp project.
 */
#ifndef COMP_B200_H
#define COMP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t; declared here so FFI users need no CUDA header. */
typedef struct CUstream_st* b2q_stream_t;

#define B2Q_OK 0
#define B2Q_EINVAL (-1)    /* bad shape / null pointer / K not a multiple of the block */
#define B2Q_EALIGN (-2)    /* pointer or stride misaligned */
#define B2Q_ECUDA (-3)     /* CUDA runtime error (launch, attribute, device query) */
#define B2Q_ERANGE (-4)    /* size beyond what this build supports (e.g. K*M too large for shared memory) */
#define B2Q_ETIMEOUT (-5)  /* a bounded device-side wait gave up (multi-GPU exchange) */

/* Weight formats and GEMV variants. Variant 0 = byte-wise unpack ("bytes"), 1/2 = packed-word dp4a ("dp4a").
 * All variants return identical int32 block dots and identical Y. Mirrors host.MODES (src/komp/host.py:13). */
#define B2Q_FMT_Q4_0 0
#define B2Q_FMT_TQ2_0 1
#define B2Q_FMT_Q8_0 2 /* extension: ggml block_q8_0 weights (no counterpart in the reference) */
#define B2Q_FMT_IQ4_NL 3 /* extension: ggml block_iq4_nl weights, GEMV path only (no counterpart in the reference) */
#define B2Q_FMT_Q4_K 4   /* extension: ggml block_q4_K weights, GEMV path only (no counterpart in the reference) */
#define B2Q_VARIANT_BYTES 0
#define B2Q_VARIANT_DP4A 2

/* Library version string, e.g. "comp_b200 0.1.0 sm_100a". */
const char* b2q_version(void);

/* Copies the calling thread's last error message into buf (always NUL-terminated); returns its full length. */
int b2q_last_error(char* buf, size_t len);

/* Number of kernels this library has launched in this process (all devices, all threads). */
long long b2q_launch_count(void);

/*
 * Activation quantizer, q8_0 (32-value blocks): per block d = amax/127 (IEEE div), id = 1/d (0 if d == 0),
 * q = roundf(x*id) with q from the unrounded f32 d, XD = f32(f16_rne(d)).
 * Replaces kernel quant_q8_0 (src/komp/kernels.py:22-33) launched by host.quantize (src/komp/host.py:63-69);
 * math of ktl.q8_0_quantize (patches/0001-language-extra-kurn.patch:104-114).
 * x: f32 [M][ldx] (first K columns used); xq: int8 [M][K]; xd: f32 [M][K/32]. K % 32 == 0.
 */
int b2q_quant_q8_0(const float* x, int64_t ldx, int8_t* xq, float* xd, int64_t M, int64_t K, b2q_stream_t stream);

/*
 * Activation quantizer, q8_K (256-value blocks): signed max-|x| (first index on ties), iscale = -127/max,
 * q = min(127, rint(iscale*x)), d = 1/iscale; all-zero block -> q = 0, d = 0.
 * Replaces kernel quant_q8_K (src/komp/kernels.py:36-45) launched by host.quantize (src/komp/host.py:70-72);
 * math of ktl.q8_K_quantize (patch:117-131). bsums (nullable) receives ggml's 16 int16 sums of 16 quants per
 * block, [M][K/256][16], which host.q8_K_blocks (src/komp/host.py:43-52) adds on the host in the reference.
 */
int b2q_quant_q8_K(const float* x, int64_t ldx, int8_t* xq, float* xd, int16_t* bsums, int64_t M, int64_t K,
                   b2q_stream_t stream);

/*
 * Q4_0 x q8_0 decode GEMV: Y[m][n] = sum_b f32(s[m][n][b]) * dw[n][b] * dx[m][b], with s the exact int32 block dot
 * sum_i (nibble_i - 8) * xq_i. Replaces kernel q4_0_gemv (src/komp/kernels.py:48-94) launched by host.gemv
 * (src/komp/host.py:76-85).
 *   wq: u8 [N][ldwq] quant plane (16 bytes per 32-value block; byte i = value i (low nibble), value i+16 (high))
 *   ws: int16 [N][K/32] f16 bit patterns of the block scales
 *   xq: int8 [M][K], xd: f32 [M][K/32]  (q8_0 split planes from b2q_quant_q8_0)
 *   y:  f32 [M][N]
 *   s:  int32 [M][N][K/32] or NULL: when given, every int32 block dot is stored (host.gemv store_s=True).
 *   variant: B2Q_VARIANT_BYTES or B2Q_VARIANT_DP4A (1 is accepted as DP4A).
 */
int b2q_gemv_q4_0(const uint8_t* wq, int64_t ldwq, const int16_t* ws, const int8_t* xq, const float* xd, float* y,
                  int32_t* s, int64_t N, int64_t K, int64_t M, int variant, b2q_stream_t stream);

/*
 * TQ2_0 x q8_K decode GEMV: Y[m][n] = sum_b dx[m][b] * dw[n][b] * f32(s[m][n][b]), s = sum_v (crumb_v - 1) * xq_v
 * where value v of a block is in quant byte (v/128)*32 + v%32 at bits 2*((v%128)/32).
 * Replaces kernel tq2_0_gemv (src/komp/kernels.py:97-142) launched by host.gemv (src/komp/host.py:76-85).
 *   wq: u8 [N][ldwq] (64 bytes per 256-value block), ws: int16 [N][K/256], xq: int8 [M][K], xd: f32 [M][K/256],
 *   y: f32 [M][N], s: int32 [M][N][K/256] or NULL.
 */
int b2q_gemv_tq2_0(const uint8_t* wq, int64_t ldwq, const int16_t* ws, const int8_t* xq, const float* xd, float* y,
                   int32_t* s, int64_t N, int64_t K, int64_t M, int variant, b2q_stream_t stream);

/*
 * Q8_0 x q8_0 decode GEMV: Y[m][n] = sum_b f32(s[m][n][b]) * dw[n][b] * dx[m][b], s = sum_i wq_i * xq_i (int8 x int8).
 * An extension beyond the reference (COMP has Q4_0 and TQ2_0 only): the weights are ggml block_q8_0 (f16 d, 32
 * int8), split like Q4_0 into a quant plane and a scale plane; the activations are the same q8_0 planes as Q4_0's.
 *   wq: u8 [N][ldwq] (the int8 values, 32 bytes per 32-value block), ws: int16 [N][K/32] (f16 bits),
 *   xq: int8 [M][K], xd: f32 [M][K/32], y: f32 [M][N], s: int32 [M][N][K/32] or NULL.
 */
int b2q_gemv_q8_0(const uint8_t* wq, int64_t ldwq, const int16_t* ws, const int8_t* xq, const float* xd, float* y,
                  int32_t* s, int64_t N, int64_t K, int64_t M, int variant, b2q_stream_t stream);

/*
 * IQ4_NL x q8_0 decode GEMV: Y[m][n] = sum_b f32(s[m][n][b]) * dw[n][b] * dx[m][b], s = sum_i level[nibble_i] * xq_i
 * with ggml's 16 int8 levels (kvalues_iq4nl: -127, -104, ..., 89, 113). A second extension beyond the reference: the
 * weights are ggml block_iq4_nl (f16 d, 16 bytes of nibbles laid out exactly as Q4_0's), so the planes are Q4_0's:
 *   wq: u8 [N][ldwq] (16 bytes per 32-value block), ws: int16 [N][K/32] (f16 bits), xq: int8 [M][K], xd: f32
 *   [M][K/32], y: f32 [M][N], s: int32 [M][N][K/32] or NULL.
 * Every fused, split-K, pinned, no-alloc and multi-GPU entry takes fmt B2Q_FMT_IQ4_NL too; layers of 8+ columns stay
 * on the GEMV path (there is no IQ4_NL tensor-core kernel).
 */
int b2q_gemv_iq4_nl(const uint8_t* wq, int64_t ldwq, const int16_t* ws, const int8_t* xq, const float* xd, float* y,
                    int32_t* s, int64_t N, int64_t K, int64_t M, int variant, b2q_stream_t stream);

/*
 * Q4_K x q8_K decode GEMV. A third extension beyond the reference: ggml block_q4_K super-blocks of 256 values, eight
 * 32-value sub-blocks with 6-bit scales sc_j and mins m_j, value = d * sc_j * q - dmin * m_j (q = 0..15), against
 * q8_K activations (the TQ2_0 activation planes). This backend's split planes (host.split("q4_k") and
 * b2q_split_blocks fmt 4 make them from the ggml blocks):
 *   wq: u8 [N][ldwq], 128 bytes per super-block: sub-block j as one 16-byte chunk laid out like a Q4_0 block (byte
 *       i: value 32j+i in the low nibble, value 32j+16+i in the high nibble);
 *   ws: int16 [N][K/256 * 10], 20 bytes per super-block: f16 d, f16 dmin, then the bytes sc_0, m_0, ..., sc_7, m_7;
 *   xq: int8 [M][K], xd: f32 [M][K/256], y: f32 [M][N], s: int32 [M][N][K/256] or NULL.
 * Y[m][n] = sum over sub-blocks of dx * (d * f32(sc_j * q.x) - dmin * f32(m_j * sum(x))); the integer parts are
 * exact, s[m][n][b] = sum_j sc_j * (q.x over sub-block j). K must be a multiple of 1024 and ws 16-byte aligned (the
 * scale records travel with the weights through the TMA ring, in whole 16-byte units); variant is ignored (one
 * kernel). Every fused, split-K, pinned, no-alloc and multi-GPU entry takes fmt B2Q_FMT_Q4_K; 8+ columns stay on the
 * GEMV path. No reference counterpart (COMP has Q4_0 and TQ2_0 only).
 */
int b2q_gemv_q4_k(const uint8_t* wq, int64_t ldwq, const int16_t* ws, const int8_t* xq, const float* xd, float* y,
                  int32_t* s, int64_t N, int64_t K, int64_t M, int variant, b2q_stream_t stream);

/*
 * Fused quantizer prologue + GEMV (one launch): every CTA quantizes f32 x into shared memory with exactly the math of
 * b2q_quant_q8_0 / b2q_quant_q8_K, then runs the GEMV. xq/xd (nullable) also receive the quantized activations
 * (written by CTA 0 only), byte-identical to the standalone quantizer. fmt = B2Q_FMT_Q4_0, B2Q_FMT_TQ2_0 or B2Q_FMT_Q8_0.
 * Fuses host.quantize + host.gemv (src/komp/host.py:63-85) into one kernel; no reference counterpart as one call.
 */
int b2q_quant_gemv(int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws, const float* x, int64_t ldx,
                   int8_t* xq, float* xd, float* y, int64_t N, int64_t K, int64_t M, b2q_stream_t stream);

/*
 * Workspace bytes b2q_quant_gemv_ws uses for this layer shape (0 = none). With M at or above the tensor-core column
 * threshold (b2q_set_gemm_min_columns; at its default from 5 columns, TQ2_0 from 3, on layers the warp-specialized
 * schedule takes) it holds the quantized activations in the MMA tile layout, and for a layer whose 128-row tiles alone
 * do not fill the GPU also the partial sums of its K ranges (the warp-specialized GEMM then splits K, and a third
 * launch adds the ranges in order). With fewer columns it is the GEMV's split-K scratch under the current split-K mode
 * (0 = the layer is not split; see b2q_set_splitk).
 * Tall-K layers (rows of more than 256 16-byte chunks, e.g. K = 14336 Q4_0 or K = 28672 TQ2_0) are split over K
 * into 2-4 independent slices computed concurrently (blockIdx.y); each writes partial sums [splits][M][N] to the
 * workspace and a second kernel sums them in split order (deterministic). Part of the north star's split-K schedule
 * for tall-K layers; no reference counterpart (COMP loops over K inside one program, kernels.py:61).
 */
size_t b2q_workspace_size(int fmt, int64_t N, int64_t K, int64_t M);

/* Split-K mode (process-wide): 0 = never split (default: on B200 the unsplit kernel measured faster on every
 * BASELINE tall-K layer), 1 = split tall-K layers automatically, n >= 2 = n splits where the shape allows. */
int b2q_set_splitk(int mode);

/*
 * b2q_quant_gemv with a caller-provided workspace (device memory, 16-byte aligned): when workspace_bytes >=
 * b2q_workspace_size(fmt, N, K, M) > 0 the split-K schedule runs; otherwise exactly b2q_quant_gemv. Two launches
 * when split (GEMV, then the combine), one otherwise. Results match b2q_quant_gemv within f32 rounding (the split
 * changes the summation order) and are deterministic. Fuses host.quantize + host.gemv (src/komp/host.py:63-85).
 */
int b2q_quant_gemv_ws(int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws, const float* x, int64_t ldx,
                      int8_t* xq, float* xd, float* y, int64_t N, int64_t K, int64_t M, void* workspace,
                      size_t workspace_bytes, b2q_stream_t stream);

/* Device workspace bytes b2q_quant_gemv_pinned needs for this layer: the staged activations (M * K f32, rounded up
 * to 256 bytes) followed by b2q_workspace_size(fmt, N, K, M). 0 for an empty layer. */
size_t b2q_pinned_workspace_size(int fmt, int64_t N, int64_t K, int64_t M);

/*
 * b2q_quant_gemv_ws with the activations and the output in page-locked host memory: x_host [M][ldx] f32 (16-byte
 * aligned, ldx % 4 == 0) and y_host [M][N] f32, both mapped for the current device (cudaHostAlloc, cudaHostRegister
 * with cudaHostRegisterMapped, torch pin_memory); anything else is refused with B2Q_EINVAL before any launch.
 * workspace: device memory, 256-byte aligned, >= b2q_pinned_workspace_size bytes. A copy kernel reads x through its
 * device mapping into the workspace, then the fused GEMV (exactly b2q_quant_gemv_ws: same schedule, bit-identical Y)
 * stores Y straight into y_host -- no memcpy, so consecutive calls keep the programmatic overlap of their kernels.
 * Asynchronous on `stream`: read y_host after synchronizing the stream. Two launches (three when the layer takes a
 * two-kernel schedule). Host-buffer form of host.quantize + host.gemv (src/komp/host.py:63-85), whose callers pass
 * torch tensors that may live on the host; no single-call counterpart in the reference.
 */
int b2q_quant_gemv_pinned(int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws, const float* x_host,
                          int64_t ldx, float* y_host, int64_t N, int64_t K, int64_t M, void* workspace,
                          size_t workspace_bytes, b2q_stream_t stream);

/*
 * The device address of page-locked host memory mapped for the current device (cudaHostAlloc, cudaHostRegister with
 * cudaHostRegisterMapped, torch pin_memory), so that a kernel of this library may store its Y there (e.g. the output
 * of b2q_gemv_allgather, which only ever writes Y). Anything else (pageable or device memory) gives B2Q_EINVAL and
 * *dev = NULL. Helper of the host-buffer paths; no reference counterpart.
 */
int b2q_host_device_pointer(const void* host, void** dev);

/*
 * Copies activations x_host [M][ldx] f32 (page-locked, mapped; 16-byte aligned, K and ldx multiples of 4) into
 * stage [M][K] (device memory, 16-byte aligned) with a kernel that reads x through its device mapping: it loads
 * before its programmatic-dependency wait and releases the next kernel at once, so a GEMV launched after it starts
 * streaming weights while x arrives (and waits for the copy before reading x). Asynchronous on `stream`. The copy
 * step of b2q_quant_gemv_pinned on its own, for callers that launch the GEMV themselves (row-sharded layers).
 */
int b2q_stage_pinned(const float* x_host, int64_t ldx, float* stage, int64_t M, int64_t K, b2q_stream_t stream);

/*
 * ggml blocks -> split planes on the device (model load path). blocks: n rows of k values as ggml Q4_0 (fmt 0,
 * 18-byte blocks: f16 d, 16 quant bytes), TQ2_0 (fmt 1, 66-byte blocks: 64 quant bytes, f16 d), Q8_0 (fmt 2,
 * 34-byte blocks: f16 d, 32 int8), IQ4_NL (fmt 3, as Q4_0) or Q4_K (fmt 4, 144-byte blocks -> the planes described at
 * b2q_gemv_q4_k: WS then holds 20 bytes per block and must be 16-byte aligned), row-major,
 * 16-byte aligned device memory (a GGUF tensor's bytes as stored). Writes WQ [n][ldwq] (ldwq >= quant bytes per row,
 * multiple of 16) and WS [n][k/blk] int16 (f16 bits), exactly host.split's planes. Replaces the host-side numpy cut
 * of src/komp/host.py:16-22 for weights already on the GPU.
 */
int b2q_split_blocks(int fmt, const uint8_t* blocks, int64_t n, int64_t k, uint8_t* wq, int64_t ldwq, int16_t* ws,
                     b2q_stream_t stream);

/*
 * Split-K fused quantize + GEMV that allocates nothing, for callers that cannot allocate device memory (an inference
 * engine that reserves all GPU memory at start-up, or an FFI caller without a device allocator of its own). It is
 * b2q_quant_gemv_ws with exactly `splits` K splits (2..16, dividing the blocks of a row) whose partial sums live in
 * a fixed scratch array inside the library: b2q_noalloc_scratch_bytes() bytes (4 MiB) on every GPU that loads the
 * library, held until the process exits. splits * M * N * 4 must fit in it (else B2Q_ERANGE), M <= 4.
 * The first call on a device, with that device current, looks up the array's device address (cudaGetSymbolAddress)
 * and keeps it for the life of the process; make that first call before any stream capture. A cudaDeviceReset (or
 * any teardown of the device's primary context) can move the array, so after one this entry point must not be used
 * again in the process. Every call shares the one array, which keeps the last call's
 * partial sums (each call overwrites all the sums it reads, so nothing has to start at zero); calls whose work
 * overlaps on the GPU (other streams, other host threads) race on it. No counterpart in the reference.
 */
size_t b2q_noalloc_scratch_bytes(void);
int b2q_quant_gemv_splitk_noalloc(int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws, const float* x,
                                  int64_t ldx, float* y, int64_t N, int64_t K, int64_t M, int splits,
                                  b2q_stream_t stream);

/*
 * Row-sharded GEMV with the output all-gather fused into the kernel (multi-GPU, one process per GPU).
 * This rank owns rows [row0, row0 + n_local) of a layer with N_total rows; wq/ws hold only those rows. The kernel
 * quantizes the replicated f32 activations x [M][ldx] in its prologue (as b2q_quant_gemv), computes its rows into
 * y [M][N_total], and sends every value to every other rank as one 64-bit scalar store of the word
 * (1 << 32 | value bits) into that rank's receive buffer (rx_peers[q], peer-mapped); a naturally aligned 64-bit access
 * is single-copy atomic, so the flag is never seen without its value. Each CTA then collects a slice of the other
 * ranks' rows from its own rx: it polls each entry (at most spin_limit times) until its flag is set, copies the value
 * into y and clears the entry. When the kernel completes, y holds all N_total rows. No fences and no grid-wide barrier
 * are needed.
 *   rx:        this rank's receive buffer, 2 x rx_stride 8-byte-aligned uint64 entries (low 32 bits: value bits,
 *              high 32 bits: flag), zeroed once before the first call; entry (m, row) of a call sits at
 *              parity * rx_stride + m*N_total + row.
 *   rx_peers:  device array [nranks] of the ranks' rx base pointers (rx_peers[rank] == rx).
 *   done:      uint64 counter of completed CTAs, zeroed once; the call index is done / grid, its parity selects
 *              the half of rx, so consecutive calls (also as CUDA-graph replays) alternate halves.
 *   status:    device int32 set to 1 if a poll gave up (the output is then invalid); the call returns B2Q_OK once
 *              launched. After status 1 the exchange state is no longer consistent (a late value may still land in
 *              rx): before the next call every rank must wait for its stream, meet the others (a host barrier), zero
 *              rx, done and status, and meet again (comp_b200.dist.RowShardedGemv.reset does this).
 *   Every rank must make the same sequence of calls with the same shapes. M <= 4.
 * No reference counterpart (the reference has no multi-GPU path); replaces host.gemv + an NCCL all-gather.
 */
int b2q_gemv_allgather(int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws, const float* x, int64_t ldx,
                       float* y, void* rx, void* const* rx_peers, int64_t rx_stride, unsigned long long* done,
                       int32_t* status, int64_t row0, int64_t n_local, int64_t N_total, int64_t K, int64_t M,
                       int rank, int nranks, long long spin_limit, b2q_stream_t stream);

/* Benchmark/tuning hook (process-wide): force rows per group (1, 2, 4), chunks per thread and grid size of the
 * GEMV schedule; 0 restores the planner's choice. Results do not depend on it (except the f32 summation order). */
int b2q_set_tuning(int rows_per_group, int chunks_per_thread, int grid);

/* Benchmark/tuning hook (process-wide): weight-streaming path 0 = planner's choice, 1 = TMA bulk-copy ring in shared
 * memory, 2 = streaming loads into registers, 5 = warp-rows schedule (one column: each warp owns whole rows and has its
 * own TMA ring); stages = ring depth (0 = planner, else 2..8). path 3 / 4 turns the programmatic dependent launch of
 * the GEMV kernels on (default) / off (stages ignored). Results do not change (except the f32 summation order). */
int b2q_set_pipeline(int path, int stages);

/* Benchmark/tuning hook (process-wide): warps per CTA of the warp-rows schedule (4..16; 0 = planner's choice). */
int b2q_set_warps(int warps);

/* Tuning hook (process-wide): layers with at least m activation columns run on the tensor-core GEMM (tcgen05 int8
 * MMA, weights read once for all columns; default 8, 0 = never). Fused calls then quantize first into the caller's
 * XQ / XD outputs or the workspace (b2q_workspace_size reports its size); int32 block dots are unchanged, Y differs
 * from the GEMV path only by the f32 summation order. At the default, a fused call with f32 activations and a workspace
 * of b2q_workspace_size bytes takes the warp-specialized tensor-core schedule from 5 columns already (TQ2_0: from 3);
 * up to 4 columns (TQ2_0: 2) the GEMV keeps every column's activation chunk in registers and reads the weights once. */
int b2q_set_gemm_min_columns(int m);

/* Tuning hook (process-wide): the fused tensor-core schedule. 0 (default) = warp-specialized where it applies (a
 * workspace of b2q_workspace_size bytes, K a whole number of 128-byte weight stages, and not the 128-column tiles
 * (M > 64) of Q4_0 / Q8_0, where the per-block schedule measured faster): a quantizing prep kernel writes
 * the activations in the MMA tile layout, then a persistent GEMM with producer, MMA and unpack/epilogue warps; 1 = the
 * per-block schedule. Identical results (same int32 dots, same f32 order), except that under the default column
 * threshold a layer too narrow to fill the GPU with its row tiles splits K on the warp-specialized schedule (its Y then
 * differs by the f32 order of adding the K ranges; the per-block schedule does not split, so such a layer stays on the
 * GEMV path without the workspace). */
int b2q_set_gemm_schedule(int schedule);

/* Benchmark/tuning hook (process-wide): ring path with one column -- the CTAs of a thread-block cluster of this size
 * (2, 4 or 8) split the activation prologue, each quantizing its share once and storing it into every member's shared
 * memory; 1 = off, 0 = planner's choice. Results do not change (identical bytes, identical summation order). */
int b2q_set_cluster(int ctas);


/* Reads (and with clear != 0 resets) the library's device error word: nonzero if a kernel's bounded wait on an
 * mbarrier gave up (the kernel then returned early; its outputs are invalid). Synchronizes with the device. */
int b2q_device_error(int* code, int clear);

/* CUDA IPC helpers for the multi-GPU path. b2q_ipc_get_handle exports the allocation containing dev_ptr as a 64-byte
 * handle and returns dev_ptr's byte offset inside it; b2q_ipc_open_handle maps a peer's allocation (with peer access
 * enabled) and returns its base, to which the peer's offset is added; b2q_ipc_close_handle unmaps that base. */
int b2q_ipc_get_handle(void* dev_ptr, void* handle_out64, uint64_t* offset_out);
int b2q_ipc_open_handle(const void* handle64, void** dev_ptr_out);
int b2q_ipc_close_handle(void* dev_ptr);

/*
 * Unit probes (test-only counterparts of the reference's probe kernels):
 *   b2q_probe_dp4a:    out[i] = c[i] + dot of the 4 signed bytes of a[i], b[i]  (kernels.py:145-149, dp4a_probe)
 *   b2q_decode_q4_0:   [R][16] quant bytes -> [R][32] int32 values nibble-8 in natural order (kernels.py:152-157)
 *   b2q_decode_tq2_0:  [R][64] quant bytes -> [R][256] int32 values crumb-1 in value order (kernels.py:160-170)
 */
int b2q_probe_dp4a(const int32_t* a, const int32_t* b, const int32_t* c, int32_t* out, int64_t n, b2q_stream_t stream);
int b2q_decode_q4_0(const uint8_t* wq, int32_t* out, int64_t R, b2q_stream_t stream);
int b2q_decode_tq2_0(const uint8_t* wq, int32_t* out, int64_t R, b2q_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* COMP_B200_H */
