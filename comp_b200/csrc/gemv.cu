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
//     order of a row depends only on (K, T, CPT), so Y is bit-identical across paths, variants, R and grid size. On
//     the ring path the issuing of the next copy and the cross-warp sum rotate over the warps group by group.
//   * Opt-in schedules: split-K over gridDim.y with an ordered combine kernel (b2q_set_splitk), and the warp-rows
//     schedule for one column (b2q_set_pipeline path 5: each warp owns whole rows and streams them through its own
//     TMA ring, activations in shared memory). Both are slower on the B200 layer shapes measured so far.
#include <algorithm>
#include <cmath>
#include <atomic>
#include <mutex>
#include <unordered_map>

#include "gemv_kernels.cuh"

namespace b2q {

// Weight formats: 0 Q4_0, 1 TQ2_0, 2 Q8_0, 3 IQ4_NL (2 and 3: extensions beyond the reference).
static inline int fmt_block(int fmt) { return (fmt == 1 || fmt == 4) ? 256 : 32; }  // values per block
static inline int fmt_chunk_values(int fmt) {                                       // per 16-byte chunk
  return (fmt == 0 || fmt == 3 || fmt == 4) ? 32 : fmt == 1 ? 64 : 16;
}
static inline int fmt_scale_bytes(int fmt) { return fmt == 4 ? 20 : 2; }  // scale-plane bytes per block
static inline bool fmt_act_q8K(int fmt) { return fmt == 1 || fmt == 4; }  // q8_K activations (else q8_0)
static inline bool fmt_ok(int fmt) { return fmt >= 0 && fmt <= 4; }
static inline size_t fmt_slot_bytes(int fmt, int C) {
  return fmt == 0 ? cluster_slot_bytes<0>(C) : fmt == 1 ? cluster_slot_bytes<1>(C)
                  : fmt == 2 ? cluster_slot_bytes<2>(C) : fmt == 3 ? cluster_slot_bytes<3>(C)
                                                                   : cluster_slot_bytes<4>(C);
}
static const char* fmt_list = "Q4_0 (0), TQ2_0 (1), Q8_0 (2), IQ4_NL (3) or Q4_K (4)";

// ------------------------------------------------------------------------------------------------------------------
// ------------------------------------------------------------------------------------------------------------------
// Host side: planning and launch
// ------------------------------------------------------------------------------------------------------------------

// Split-K combine: y[m][n] = sum over s of partial[s][m][n], splits summed in order 0, 1, ... (deterministic).
// Launched with programmatic stream serialization after the split GEMV; reads the partials only after the wait.
__global__ void __launch_bounds__(256) splitk_sum_kernel(const float* __restrict__ partial, float* __restrict__ y,
                                                         int64_t M, int64_t N, int64_t ldy, int splits) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int64_t total = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    float v = partial[i];
    for (int s = 1; s < splits; ++s) v += partial[(int64_t)s * total + i];
    const int64_t m = i / N, n = i - m * N;
    y[m * ldy + n] = v;
  }
}

static KernelFn kernel_for(int fmt, bool bytes, bool ring, int R, int MC, bool xreg) {
  return ring ? ring_kernel_for(fmt, R, MC, xreg) : reg_kernel_for(fmt, bytes, R, MC, xreg);
}

struct OccKey {
  int dev;
  KernelFn fn;
  int threads;
  size_t smem;
  bool operator==(const OccKey& o) const {
    return dev == o.dev && fn == o.fn && threads == o.threads && smem == o.smem;
  }
};
struct OccHash {
  size_t operator()(const OccKey& k) const {
    return std::hash<const void*>()((const void*)k.fn) ^ (k.threads * 131u) ^ (k.smem * 7919u) ^ (k.dev * 31u);
  }
};
static std::mutex g_occ_mu;
static std::unordered_map<OccKey, int, OccHash> g_occ;

// Resident CTAs per SM for this kernel and launch shape (opts the kernel into large dynamic shared memory first).
static int occupancy(KernelFn fn, int threads, size_t smem, int max_smem_optin) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  OccKey key{dev, fn, threads, smem};
  {
    std::lock_guard<std::mutex> lk(g_occ_mu);
    auto it = g_occ.find(key);
    if (it != g_occ.end()) return it->second;
  }
  cudaFuncAttributes attr;
  if (cudaFuncGetAttributes(&attr, (const void*)fn) != cudaSuccess) return -1;
  if (smem + attr.sharedSizeBytes > (size_t)max_smem_optin) return 0;
  if (cudaFuncSetAttribute((const void*)fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           max_smem_optin - (int)attr.sharedSizeBytes) != cudaSuccess)
    return -1;
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, (const void*)fn, threads, smem) != cudaSuccess)
    return -1;
  std::lock_guard<std::mutex> lk(g_occ_mu);
  g_occ[key] = blocks;
  return blocks;
}

// Process-wide tuning state below is written by the b2q_set_* hooks and read by every launch: atomics, so a hook
// called from one host thread while another launches is no data race (that launch sees the old or the new setting;
// results are the same either way, up to the f32 summation order of a different schedule).

// Programmatic dependent launch of the GEMV kernels (on by default; b2q_set_pipeline path 3/4 toggles it).
static std::atomic<int> g_pdl{1};
bool pdl_enabled() { return g_pdl != 0; }

// Tuning overrides (benchmark hook): 0 = planner's choice.
static std::atomic<int> g_tune_rows{0}, g_tune_cpt{0}, g_tune_grid{0}, g_tune_stages{0}, g_tune_path{0};

struct Plan {
  int R, T, CPT, grid, stages;
  uint32_t stage_bytes;
  size_t smem;
  bool ring;
  KernelFn fn;
  int cluster = 1;  // CTAs per thread-block cluster sharing the activation prologue (ring path, one column)
};

// CTAs per cluster for the shared activation prologue: 0 = planner, 1 = off, 2 / 4 / 8 = forced. The planner uses
// pairs whenever every CTA slot of the grid can still be filled by whole clusters, except for short TQ2_0 rows (see
// make_plan_uncached): measured on B200, pairs win on K = 28672 rows and on the Q4_0 lm_head (88 vs 96 us), lose on
// K = 8192 TQ2_0 rows since the register prologue got cheaper; clusters of 4 or 8 lose everywhere.
static std::atomic<int> g_tune_cluster{0};

// Clusters of `cs` CTAs of this kernel and launch shape that can be resident at once on the device.
static int max_active_clusters(KernelFn fn, int threads, size_t smem, int cs) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)cs);
  cfg.blockDim = dim3((unsigned)threads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute a[1];
  a[0].id = cudaLaunchAttributeClusterDimension;
  a[0].val.clusterDim.x = (unsigned)cs;
  a[0].val.clusterDim.y = 1;
  a[0].val.clusterDim.z = 1;
  cfg.attrs = a;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, (const void*)fn, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

// Shared memory besides the ring: staged activations (none when they live in registers) and the reduction partials.
static size_t x_region_bytes(int fmt, int64_t K, int M, int C, int R, int MC, int T, bool xreg) {
  const int nblk = (int)(K / fmt_block(fmt));
  const int Mx = xreg ? 0 : M;
  return (size_t)Mx * K + (size_t)Mx * C * 4 + (size_t)Mx * nblk * 4 + (size_t)2 * (T / 32) * R * MC * 4;
}

static uint32_t ring_stage_bytes(int fmt, int64_t K, int C, int R) {
  const int nblk = (int)(K / fmt_block(fmt));
  const uint32_t s = (uint32_t)R * (uint32_t)nblk * (uint32_t)fmt_scale_bytes(fmt);
  return (uint32_t)R * (uint32_t)C * 16u + ((s + 15u) & ~15u);
}

// Plans depend only on the device, the layer shape and the tuning hooks, so each is computed once: the occupancy
// queries behind a plan cost host time that a decode loop, which waits for every step's result, would otherwise pay
// before every first launch of a step.
struct PlanKey {
  int dev, fmt, M, splits;
  bool bytes, ring_ok;
  int64_t N, K;
  int tune[6];
  bool operator==(const PlanKey& o) const {
    return dev == o.dev && fmt == o.fmt && M == o.M && splits == o.splits && bytes == o.bytes &&
           ring_ok == o.ring_ok && N == o.N && K == o.K && std::equal(tune, tune + 6, o.tune);
  }
};
struct PlanHash {
  size_t operator()(const PlanKey& k) const {
    size_t h = std::hash<int64_t>()(k.N) * 1000003u ^ std::hash<int64_t>()(k.K);
    h = h * 31u + (size_t)(k.dev * 7 + k.fmt) * 131u + (size_t)k.M * 17u + (size_t)k.splits;
    h = h * 31u + (k.bytes ? 1u : 0u) + (k.ring_ok ? 2u : 0u);
    for (int t : k.tune) h = h * 31u + (size_t)t;
    return h;
  }
};
static std::mutex g_plan_mu;
static std::unordered_map<PlanKey, Plan, PlanHash> g_plans;

static int make_plan_uncached(int fmt, bool bytes, bool ring_ok, int64_t N, int64_t K, int M, Plan* out, int splits);

// K is the per-split K; `splits` CTAs rows share the SMs (the grid is splits x grid_x).
static int make_plan(int fmt, bool bytes, bool ring_ok, int64_t N, int64_t K, int M, Plan* out, int splits = 1) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(B2Q_ECUDA, "gemv: cudaGetDevice failed");
  const PlanKey key{dev, fmt, M, splits, bytes, ring_ok, N, K,
                    {g_tune_rows, g_tune_cpt, g_tune_grid, g_tune_stages, g_tune_path, g_tune_cluster}};
  {
    std::lock_guard<std::mutex> lk(g_plan_mu);
    auto it = g_plans.find(key);
    if (it != g_plans.end()) {
      *out = it->second;
      return B2Q_OK;
    }
  }
  const int rc = make_plan_uncached(fmt, bytes, ring_ok, N, K, M, out, splits);
  if (rc == B2Q_OK) {
    std::lock_guard<std::mutex> lk(g_plan_mu);
    g_plans[key] = *out;
  }
  return rc;
}

static int make_plan_uncached(int fmt, bool bytes, bool ring_ok, int64_t N, int64_t K, int M, Plan* out, int splits) {
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  const int C = (int)(K / fmt_chunk_values(fmt));
  int CPT = (C + kMaxThreads - 1) / kMaxThreads;
  if (g_tune_cpt > 0) CPT = g_tune_cpt;
  const int T = std::min(kMaxThreads, ((C + CPT - 1) / CPT + 31) / 32 * 32);
  if ((int64_t)T * CPT < C)
    return fail(B2Q_ERANGE, "gemv: K=%lld needs more than %d chunks per thread", (long long)K, CPT);
  // Q4_K has a ring kernel only: its byte-wise variant is the dp4a kernel (identical results)
  bool use_ring = ring_ok && (!bytes || fmt == 4) && (g_tune_path != 2 || fmt == 4);
  if (g_tune_path == 1 && !use_ring) return fail(B2Q_EINVAL, "gemv: ring path forced but not applicable");
  Plan best{};
  double best_score = -1.0;
  const int cand[5] = {16, 8, 4, 2, 1};
  for (int pass = 0; pass < 2 && best_score < 0; ++pass) {
    const bool ring = use_ring && pass == 0;
    if (pass == 1 && (g_tune_path == 1 || fmt == 4)) break;  // Q4_K: ring only
    // one chunk per thread: the activations in registers (XREG), for one column, or on the ring path for two to four
    // (each thread holds its chunk of every column: no shared-memory staging; TQ2_0 only for two, its 64-value
    // chunks spill at four); otherwise staged in shared memory, 4 columns per pass
    const bool xreg = CPT == 1 && (M == 1 || (ring && (M == 2 || (M <= 4 && fmt != 1))));
    const int MC = M == 1 ? 1 : (xreg && M == 2) ? 2 : kMaxColumns;
    for (int ci = 0; ci < 5; ++ci) {
      const int R = cand[ci];
      if (g_tune_rows > 0 && R != g_tune_rows) continue;
      // 16-row groups: ring path, one column, one chunk per thread, CTAs of at most 256 threads. Measured on B200:
      // TQ2_0 gate_up 2% faster than 8 rows, Q4_0 lm_head unchanged -- so TQ2_0 by default, Q4_0 on request.
      if (R == 16 && (!ring || !xreg || MC != 1 || T > 256 || (fmt != 1 && g_tune_rows != 16))) continue;
      if (xreg && MC == 4 && R > 4 && fmt != 2) continue;  // the four-column register kernels spill above 4 rows
      const size_t xb = x_region_bytes(fmt, K, M, C, R, MC, T, xreg);
      const int64_t groups = (N + R - 1) / R;
      int stages = 0;
      uint32_t sb = 0;
      size_t smem = xb;
      if (ring) {
        // Measured on B200 (weight-streaming sweeps over the BASELINE layer shapes): two stages -- one group in
        // flight while one is computed -- with the most CTAs per SM beats deeper rings at lower occupancy.
        sb = ring_stage_bytes(fmt, K, C, R);
        stages = g_tune_stages > 0 ? g_tune_stages.load() : 2;
        smem = (size_t)stages * sb + 8 * (size_t)((stages + 1) & ~1) + xb;
      }
      int cs = 1;
      // pairs by default, except TQ2_0 rows of at most 128 chunks (K <= 8192), where each CTA's own prologue is
      // short and the pair's exchange and barrier cost more than they save (measured on B200: gate_up 57344x8192
      // 23.6 vs 24.3 us, its 8-GPU slice 7168x8192 6.3 vs 7.5 us; K = 28672 rows and Q4_0 keep pairs)
      const int auto_cs = (fmt == 1 && C <= 128) ? 1 : 2;
      if (ring && xreg && MC == 1)
        cs = g_tune_cluster > 1 ? g_tune_cluster.load() : (g_tune_cluster == 0 ? auto_cs : 1);
      const size_t slot = fmt_slot_bytes(fmt, C);
      if (cs > 1 && smem + slot > (size_t)di.max_smem_optin && g_tune_cluster == 0) cs = 1;
      if (cs > 1) smem += slot;
      if (smem > (size_t)di.max_smem_optin) continue;
      KernelFn fn = kernel_for(fmt, bytes, ring, R, MC, xreg);
      int occ = occupancy(fn, T, smem, di.max_smem_optin);
      if (occ < 0) return fail(B2Q_ECUDA, "gemv: occupancy query failed: %s", cudaGetErrorString(cudaGetLastError()));
      if (cs > 1 && g_tune_cluster == 0) {  // pairs only if they cost no resident CTA
        const size_t smem1 = smem - slot;
        const int occ1 = occupancy(fn, T, smem1, di.max_smem_optin);
        const int ncl = occ > 0 ? max_active_clusters(fn, T, smem, cs) : 0;
        if (occ1 < 0) return fail(B2Q_ECUDA, "gemv: occupancy query failed");
        if (occ < occ1 || (int64_t)ncl * cs < (int64_t)occ * di.sms) {
          cs = 1;
          smem = smem1;
          occ = occ1;
        }
      }
      if (occ == 0) continue;
      int64_t grid = std::min<int64_t>(groups, std::max<int64_t>(1, (int64_t)occ * di.sms / splits));
      if (g_tune_grid > 0) grid = std::min<int64_t>(groups, g_tune_grid);
      if (cs > 1) {  // whole clusters, no more than can be resident at once (a member may own no group)
        const int ncl = max_active_clusters(fn, T, smem, cs);
        if (ncl <= 0) continue;
        grid = std::min<int64_t>(grid, (int64_t)ncl * cs / splits);
        grid = std::max<int64_t>(cs, grid / cs * cs);
      }
      // balance: groups per CTA is floor or ceil of groups/grid; efficiency = mean / max
      const int64_t per = (groups + grid - 1) / grid;
      const double balance = (double)groups / (double)(per * grid);
      // larger groups amortize the per-group reduction and barrier (measured on B200: R = 8 fastest whenever it
      // fits, even at 13% worse balance)
      const double score = balance + 0.2 * std::log2((double)R);
      if (score > best_score) {
        best_score = score;
        best = Plan{R, T, CPT, (int)grid, stages, sb, smem, ring, fn, cs};
      }
    }
  }
  if (best_score < 0)
    return fail(B2Q_ERANGE, "gemv: K=%lld with %d columns does not fit in shared memory (%d bytes max)",
                (long long)K, M, di.max_smem_optin);
  *out = best;
  return B2Q_OK;
}

// Warp-rows path (one column): W warps per CTA, one CTA per SM, each warp with its own S-stage ring of R-row groups.
static std::atomic<int> g_tune_warps{0};

static int make_warp_plan(int fmt, int64_t N, int64_t K, Plan* out) {
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  const int C = (int)(K / fmt_chunk_values(fmt));
  const int nblk = (int)(K / fmt_block(fmt));
  const size_t xbytes = (size_t)K + 4 * (size_t)C + 4 * (size_t)nblk;
  const int rows[3] = {4, 2, 1}, stages[3] = {3, 2, 4};
  double best_score = -1.0;
  Plan best{};
  for (int R : rows) {
    if (g_tune_rows > 0 && R != g_tune_rows) continue;
    const uint32_t sb = ring_stage_bytes(fmt, K, C, R);
    for (int S : stages) {
      if (g_tune_stages > 0 && S != g_tune_stages) continue;
      for (int W = kMaxThreads / 32; W >= 4; --W) {
        if (g_tune_warps > 0 && W != g_tune_warps) continue;
        const size_t smem = (size_t)W * S * sb + 8 * (size_t)((W * S + 1) & ~1) + xbytes;
        if (smem > (size_t)di.max_smem_optin) continue;
        KernelFn fn = warp_kernel_for(fmt, R);
        if (!fn) continue;
        const int occ = occupancy(fn, 32 * W, smem, di.max_smem_optin);
        if (occ < 0) return fail(B2Q_ECUDA, "gemv: occupancy query failed: %s", cudaGetErrorString(cudaGetLastError()));
        if (occ == 0) continue;
        const int64_t groups = (N + R - 1) / R;
        // more warps first (latency hiding), then larger groups (fewer reductions per row), then deeper rings
        const double score = W * 100.0 + R * 10.0 + (S == 3 ? 2 : S == 2 ? 1 : 0);
        if (score > best_score) {
          best_score = score;
          best = Plan{R, 32 * W, (C + 31) / 32, (int)std::min<int64_t>(groups, di.sms), S, sb, smem, true, fn};
        }
        break;  // the largest W that fits for this (R, S)
      }
    }
  }
  if (best_score < 0) return fail(B2Q_ERANGE, "gemv: K=%lld does not fit the warp-rows schedule", (long long)K);
  *out = best;
  return B2Q_OK;
}

// K splits the split-K schedule uses for a layer (1 = none). Off by default: on B200 the BASELINE tall-K layers ran
// slower split (TQ2_0 8192x28672: 23.4 vs 19.0 us; Q4_0 4096x14336: 14.6 vs 11.9 us) -- the unsplit kernel already
// keeps the HBM stream busy and the combine adds a launch. With b2q_set_splitk(1) tall-K layers whose rows would
// need CTAs of more than 256 threads are split until each split's row fits 256 threads; b2q_set_splitk(n) forces n.
// Every split keeps 16-byte aligned whole scale rows (ring path) and whole quads of TQ2_0 chunks. One column group
// (M <= 4) only.
static std::atomic<int> g_splitk_mode{0};  // 0: never split (default; measured slower on B200), 1: automatic rule, n>=2: force n

static int choose_splits(int fmt, int64_t K, int64_t M) {
  if (g_splitk_mode == 0 || M < 1 || M > kMaxColumns || K == 0) return 1;
  if (fmt == 4 && (K / 256) % 4) return 1;  // Q4_K: every split must keep whole 16-byte units of scale records
  const int blk = fmt_block(fmt);
  const int64_t nblk = K / blk, C = K / fmt_chunk_values(fmt);
  if (C <= 256) return 1;
  for (int s = 2; s <= 16; s *= 2) {
    if (nblk % s) continue;
    const int64_t nblk_s = nblk / s;
    if ((nblk_s * fmt_scale_bytes(fmt)) % 16) continue;
    if (g_splitk_mode >= 2 ? s == g_splitk_mode : C / s <= 256) return s;
  }
  return 1;
}

static int check_gemv_args(const char* who, int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws,
                           const void* x, const float* xd, const float* y, int64_t N, int64_t K, int64_t M,
                           bool f32_input) {
  const int blk = fmt_block(fmt);
  if (N < 0 || K < 0 || M < 0) return fail(B2Q_EINVAL, "%s: negative size", who);
  if (K % blk) return fail(B2Q_EINVAL, "%s: K=%lld is not a multiple of the %d-value block", who, (long long)K, blk);
  if (N == 0 || M == 0) return B2Q_OK;  // empty output: no pointer is touched
  if (!y) return fail(B2Q_EINVAL, "%s: null pointer", who);
  if (!aligned(y, 4)) return fail(B2Q_EALIGN, "%s: y must be 4-byte aligned", who);
  if (K == 0) return B2Q_OK;  // empty sums: only Y (= 0) is written
  if (!wq || !ws || !x || (!f32_input && !xd)) return fail(B2Q_EINVAL, "%s: null pointer", who);
  const int64_t qbytes = (fmt == 0 || fmt == 3 || fmt == 4) ? K / 2 : fmt == 1 ? K / 4 : K;
  if (ldwq < qbytes) return fail(B2Q_EINVAL, "%s: ldwq=%lld < %lld quant bytes per row", who, (long long)ldwq,
                                 (long long)qbytes);
  if (!aligned(wq, 16) || (ldwq % 16)) return fail(B2Q_EALIGN, "%s: wq must be 16-byte aligned, ldwq %% 16 == 0", who);
  if (!aligned(ws, 2)) return fail(B2Q_EALIGN, "%s: ws must be 2-byte aligned", who);
  // Q4_K runs on the TMA ring only: its 20-byte scale records must form whole 16-byte units per row
  if (fmt == 4 && (((K / 256) * 20) % 16 || !aligned(ws, 16)))
    return fail(B2Q_EALIGN, "%s: Q4_K needs K a multiple of 1024 and ws 16-byte aligned", who);
  if (!aligned(x, 16)) return fail(B2Q_EALIGN, "%s: activations must be 16-byte aligned", who);
  if (xd && !aligned(xd, 4)) return fail(B2Q_EALIGN, "%s: xd must be 4-byte aligned", who);
  if (K > (int64_t)1 << 30 || N > ((int64_t)1 << 40)) return fail(B2Q_ERANGE, "%s: size too large", who);
  return B2Q_OK;
}

int check_quant_gemv_args(const char* who, int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws, const float* x,
                          const float* y, int64_t N, int64_t K, int64_t M) {
  if (!fmt_ok(fmt)) return fail(B2Q_EINVAL, "%s: fmt %d is not %s", who, fmt, fmt_list);
  return check_gemv_args(who, fmt, wq, ldwq, ws, x, nullptr, y, N, K, M, true);
}

struct LaunchArgs {
  int fmt;
  bool bytes;
  const uint8_t* wq;
  int64_t ldwq;
  const int16_t* ws;
  const int8_t* xq;
  const float* xd;
  const float* x_f32;
  int64_t ldx;
  int8_t* xq_out;
  float* xd_out;
  float* y;
  int64_t ldy;
  int64_t row0;
  int32_t* s;
  unsigned long long* const* rx_peers;
  unsigned long long* rx;
  int64_t rx_stride;
  unsigned long long* done;
  int32_t* status;
  int rank, nranks;
  long long spin_limit;
  int64_t N, K, M;
  float* workspace;  // split-K partial sums (null: no split)
  size_t workspace_bytes;
  int force_splits;  // > 1: run exactly this many K splits (validated by the caller)
};

// Tensor-core GEMM for many columns (gemm_tc.cu): pre-quantized activations, M >= the threshold below.
int launch_gemm_tc(const GemvParams& base, int fmt, cudaStream_t stream, bool pdl);

// Warp-specialized persistent tensor-core GEMM with its quantizing prep kernel (gemm_tc_ws.cu): the fused path's
// schedule when the workspace holds its activation tiles (gemm_tc_ws_bytes > 0: K a whole number of stages).
// Layers whose row tiles alone do not fill the GPU split K (gemm_tc_ws_splits), their partial sums in the workspace.
int gemm_tc_ws_splits(int fmt, int64_t N, int64_t K, int64_t M);
size_t gemm_tc_ws_bytes(int fmt, int64_t N, int64_t K, int64_t M, int ks);
int launch_gemm_tc_ws(int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws, const float* x, int64_t ldx,
                      int8_t* xq_out, float* xd_out, float* y, int64_t ldy, int64_t row0, int64_t N, int64_t K,
                      int64_t M, int ks, void* workspace, cudaStream_t stream, bool pdl);

// Columns from which a layer runs on the tensor-core GEMM (0 = never). Below it the GEMV kernels, which re-read the
// weights per group of 4 columns, are the better fit.
static std::atomic<int> g_tc_min_m{8};
// Under the default threshold, fused calls that can take the warp-specialized schedule (a workspace, f32 activations)
// already do from this many columns. Measured on B200 (same box, us): the GEMV's register path (each thread holds its
// chunk of every column) at M = 2 / 3 / 4 against the tensor cores: Q4_0 lm_head 128256x8192 97 / 162 / 185 vs 203,
// Q8_0 lm_head 128256x4096 79 / 87 / 95 vs 139, and from M = 5 (staged in shared memory again) 273 vs 203, 174 vs 139;
// TQ2_0 (whose four-column register kernels spill) gate_up 57344x8192 at M = 2 / 3: 38 / 133 vs 83, down 8192x28672
// 24 / 82 vs 44 (K split). So TQ2_0 from 3 columns, the other formats from 5. The per-block schedule keeps the
// threshold.
static int ws_min_columns(int fmt) { return fmt == 1 ? 3 : 5; }
// Fused tensor-core schedule: 0 = warp-specialized where it applies (default), 1 = always the per-block schedule
static std::atomic<int> g_tc_schedule{0};

// Scratch for the quantized activations when a fused call takes the tensor-core path: XQ [M][K], then XD (per-block
// schedule), or the warp-specialized schedule's activation tiles -- whichever is larger.
// K splits of the warp-specialized schedule: only under the default column threshold (a lowered one is how the
// tests force the tensor-core kernels onto narrow layers, where the two schedules must agree bit for bit)
static int tc_splits(int fmt, int64_t N, int64_t K, int64_t M) {
  return g_tc_min_m.load() >= 8 ? gemm_tc_ws_splits(fmt, N, K, M) : 1;
}

static size_t tc_act_bytes(int fmt, int64_t N, int64_t K, int64_t M) {
  const int64_t nblk = K / fmt_block(fmt);
  const size_t v1 = ((size_t)M * (size_t)K + 15) / 16 * 16 + (size_t)M * (size_t)nblk * sizeof(float);
  return std::max(v1, gemm_tc_ws_bytes(fmt, N, K, M, tc_splits(fmt, N, K, M)));
}

static int launch_gemv(const LaunchArgs& a, cudaStream_t stream) {
  if (a.N == 0 || a.M == 0 || a.K == 0) {
    // empty reductions: Y = 0 (K == 0); nothing to do for N == 0 or M == 0
    if (a.K == 0 && a.N > 0 && a.M > 0) {
      cudaError_t e = cudaMemset2DAsync(a.y + a.row0, (size_t)a.ldy * 4, 0, (size_t)a.N * 4, (size_t)a.M, stream);
      if (e != cudaSuccess) return fail(B2Q_ECUDA, "gemv: cudaMemset2DAsync: %s", cudaGetErrorString(e));
    }
    return B2Q_OK;
  }
  const int blk = fmt_block(a.fmt);
  const int64_t nblk = a.K / blk;
  // many columns: the tensor-core GEMM, on pre-quantized activations (a fused call quantizes first into the caller's
  // XQ / XD outputs or the workspace; without either it stays on the GEMV path)
  // (only when its CTAs -- 128 rows x up to 128 columns each -- fill the GPU: on narrow layers the GEMV path is faster)
  DeviceInfo tc_di;
  const int tc_nt = a.M <= 16 ? 16 : a.M <= 32 ? 32 : a.M <= 64 ? 64 : 128;
  const int64_t tc_tiles = ((a.N + 127) / 128) * ((a.M + tc_nt - 1) / tc_nt);
  const bool tc_wide = device_info(&tc_di) == B2Q_OK && tc_tiles >= (int64_t)tc_di.sms;
  // narrower layers: the warp-specialized schedule with K split so that its tiles fill the GPU (when it applies)
  const int tc_ks = tc_wide ? 1 : tc_splits(a.fmt, a.N, a.K, a.M);
  const bool tc_split = !tc_wide && tc_ks > 1 && tc_tiles * tc_ks >= (int64_t)tc_di.sms;
  const int tc_min = g_tc_min_m.load();
  const bool ws_call = a.x_f32 && !a.s && g_tc_schedule == 0 && a.workspace && aligned(a.workspace, 16) &&
                       aligned(a.ws, 16) && aligned(a.x_f32, 16) && a.ldx % 4 == 0;
  const int tc_from = (tc_min == 8 && ws_call) ? ws_min_columns(a.fmt) : tc_min;  // columns from which TC applies
  // (IQ4_NL and Q4_K have no tensor-core kernel: their many-column layers stay on the GEMV path)
  if (tc_min > 0 && a.M >= tc_from && (tc_wide || tc_split || tc_min < 8) && !a.rx_peers && aligned(a.wq, 16) &&
      a.ldwq % 16 == 0 && a.fmt != 3 && a.fmt != 4) {
    const int8_t* xq = a.xq;
    const float* xd = a.xd;
    // Measured on B200 (same box, lm_head-sized layers, M = 16..128): the warp-specialized schedule is faster everywhere
    // except 128-column tiles of the 32-value block formats (Q4_0 1683 vs 1493 us, Q8_0 907 vs 772 us at M = 128),
    // where the per-block kernel stays; TQ2_0 keeps it at every width (198 vs 439 us at M = 128).
    const bool ws_fits = !(tc_nt == 128 && a.fmt != 1);
    if (ws_call && ws_fits) {
      const int ks = tc_wide ? 1 : tc_ks;
      const size_t wsb = gemm_tc_ws_bytes(a.fmt, a.N, a.K, a.M, ks);
      if (wsb && a.workspace_bytes >= wsb)
        return launch_gemm_tc_ws(a.fmt, a.wq, a.ldwq, a.ws, a.x_f32, a.ldx, a.xq_out, a.xd_out, a.y, a.ldy, a.row0,
                                 a.N, a.K, a.M, ks, a.workspace, stream, g_pdl != 0);
    }
    // the per-block kernel below cannot split K: a narrow layer that the split schedule could not take stays on the
    // GEMV path
    const bool per_block_ok = (tc_wide || tc_min < 8) && a.M >= tc_min;
    if (a.x_f32 && per_block_ok) {
      int8_t* qo = a.xq_out;
      float* dq = a.xd_out;
      if (!qo && a.workspace && a.workspace_bytes >= tc_act_bytes(a.fmt, a.N, a.K, a.M)) {
        qo = reinterpret_cast<int8_t*>(a.workspace);
        dq = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(a.workspace) + ((size_t)a.M * a.K + 15) / 16 * 16);
      }
      if (qo) {
        const int rc = !fmt_act_q8K(a.fmt) ? b2q_quant_q8_0(a.x_f32, a.ldx, qo, dq, a.M, a.K, stream)
                                  : b2q_quant_q8_K(a.x_f32, a.ldx, qo, dq, nullptr, a.M, a.K, stream);
        if (rc) return rc;
        xq = qo;
        xd = dq;
      }
    }
    if (xq && per_block_ok) {
      GemvParams p{};
      p.wq = a.wq;
      p.ldwq = a.ldwq;
      p.ws = a.ws;
      p.ldws = nblk;
      p.xq = xq;
      p.ldxq = a.K;
      p.xd = xd;
      p.ldxd = nblk;
      p.y = a.y;
      p.ldy = a.ldy;
      p.row0 = a.row0;
      p.s = a.s;
      p.N = a.N;
      p.K = a.K;
      p.M = (int)a.M;
      return launch_gemm_tc(p, a.fmt, stream, g_pdl != 0);
    }
  }
  // split-K when a workspace for the partial sums is given and the layer is tall (one column group only)
  int splits = 1;
  if (a.workspace && !a.s && !a.rx_peers && a.M <= kMaxColumns) {
    const int sp = a.force_splits > 1 ? a.force_splits : choose_splits(a.fmt, a.K, a.M);
    if (sp > 1 && (size_t)sp * a.M * a.N * sizeof(float) <= a.workspace_bytes) splits = sp;
  }
  const int64_t Ks = a.K / splits, nblk_s = nblk / splits;
  const int C = (int)(Ks / fmt_chunk_values(a.fmt));
  // ring path: every row's scale bytes (and so every group's) must be a whole number of 16-byte units, 16-aligned
  const int sbytes = fmt_scale_bytes(a.fmt);
  const bool ring_ok = ((nblk * sbytes) % 16 == 0) && ((nblk_s * sbytes) % 16 == 0) && aligned(a.ws, 16);
  if (a.fmt == 4 && !ring_ok)
    return fail(B2Q_EINVAL, "gemv: Q4_K runs on the TMA ring only: K (and each split's K) a multiple of 1024, ws "
                            "16-byte aligned");
  for (int64_t m0 = 0; m0 < a.M; m0 += kMaxColumns) {
    const int Mc = (int)std::min<int64_t>(kMaxColumns, a.M - m0);
    Plan pl;
    const bool warp_ok = Mc == 1 && a.M == 1 && splits == 1 && !a.rx_peers && ring_ok && !a.bytes && a.fmt != 4;
    if (g_tune_path == 5 && !warp_ok) return fail(B2Q_EINVAL, "gemv: warp-rows path forced but not applicable");
    int rc = (warp_ok && g_tune_path == 5) ? make_warp_plan(a.fmt, a.N, Ks, &pl)
                                           : make_plan(a.fmt, a.bytes, ring_ok, a.N, Ks, Mc, &pl, splits);
    if (rc) return rc;
    GemvParams p{};
    p.wq = a.wq;
    p.ldwq = a.ldwq;
    p.ws = a.ws;
    p.ldws = nblk * (fmt_scale_bytes(a.fmt) / 2);
    p.xq = a.xq ? a.xq + m0 * a.K : nullptr;
    p.ldxq = a.K;
    p.xd = a.xd ? a.xd + m0 * nblk : nullptr;
    p.ldxd = nblk;
    p.x_f32 = a.x_f32 ? a.x_f32 + m0 * a.ldx : nullptr;
    p.ldx = a.ldx;
    p.xq_out = a.xq_out ? a.xq_out + m0 * a.K : nullptr;
    p.xd_out = a.xd_out ? a.xd_out + m0 * nblk : nullptr;
    if (splits > 1) {  // partial sums [splits][Mc][N] in the workspace, combined below
      p.y = a.workspace;
      p.ldy = a.N;
      p.row0 = 0;
      p.y_split = (int64_t)Mc * a.N;
    } else {
      p.y = a.y + m0 * a.ldy;
      p.ldy = a.ldy;
      p.row0 = a.row0;
      p.y_split = 0;
    }
    p.s = a.s ? a.s + m0 * a.N * nblk : nullptr;
    p.rx_peers = a.rx_peers;  // the exchange path is limited to one column group (M <= kMaxColumns) by its entry point
    p.rx = a.rx;
    p.rx_stride = a.rx_stride;
    p.done = a.done;
    p.N_total = a.rx_peers ? a.ldy : a.N;
    p.status = a.status;
    p.rank = a.rank;
    p.nranks = a.nranks;
    p.spin_limit = a.spin_limit;
    p.N = a.N;
    p.K = Ks;
    p.M = Mc;
    p.C = C;
    p.CPT = pl.CPT;
    p.groups = (a.N + pl.R - 1) / pl.R;
    p.stages = pl.stages;
    p.stage_bytes = pl.stage_bytes;
    p.dense = (splits == 1 && a.ldwq == (int64_t)C * 16) ? 1 : 0;
    p.cluster = pl.cluster;
    // programmatic stream serialization: the kernel's weight prefetch may overlap the preceding kernel's tail
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)pl.grid, (unsigned)splits);
    cfg.blockDim = dim3((unsigned)pl.T);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = g_pdl ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)pl.cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pl.cluster > 1 ? 2 : 1;
    cudaError_t le = cudaLaunchKernelEx(&cfg, pl.fn, p);
    if (le != cudaSuccess) {
      cudaGetLastError();
      return fail(B2Q_ECUDA, "gemv: launch failed: %s", cudaGetErrorString(le));
    }
    rc = after_launch(a.fmt == 0   ? "gemv_q4_0"
                      : a.fmt == 1 ? "gemv_tq2_0"
                      : a.fmt == 2 ? "gemv_q8_0"
                      : a.fmt == 3 ? "gemv_iq4_nl"
                                   : "gemv_q4_k");
    if (rc) return rc;
    if (splits > 1) {
      DeviceInfo di;
      if ((rc = device_info(&di))) return rc;
      const int64_t total = (int64_t)Mc * a.N;
      cudaLaunchConfig_t c2 = {};
      c2.gridDim = dim3((unsigned)std::min<int64_t>((total + 255) / 256, (int64_t)di.sms * 4));
      c2.blockDim = dim3(256);
      c2.stream = stream;
      c2.attrs = attr;
      c2.numAttrs = 1;
      le = cudaLaunchKernelEx(&c2, splitk_sum_kernel, (const float*)a.workspace, a.y + m0 * a.ldy + a.row0,
                              (int64_t)Mc, a.N, a.ldy, splits);
      if (le != cudaSuccess) {
        cudaGetLastError();
        return fail(B2Q_ECUDA, "gemv: split-K combine launch failed: %s", cudaGetErrorString(le));
      }
      rc = after_launch("splitk_sum");
      if (rc) return rc;
    }
  }
  return B2Q_OK;
}

// Fused quantize + split-K GEMV into a given workspace with exactly `splits` K splits (used by gemv_noalloc.cu).
int quant_gemv_forced_split(int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws, const float* x, int64_t ldx,
                            float* y, int64_t N, int64_t K, int64_t M, int splits, float* workspace,
                            size_t workspace_bytes, cudaStream_t stream) {
  const char* who = "b2q_quant_gemv_splitk_noalloc";
  int rc = check_gemv_args(who, fmt, wq, ldwq, ws, x, nullptr, y, N, K, M, true);
  if (rc) return rc;
  if (M > kMaxColumns) return fail(B2Q_ERANGE, "%s: M=%lld, at most %d columns", who, (long long)M, kMaxColumns);
  const int blk = fmt_block(fmt);
  const int64_t nblk = K / blk;
  if (splits < 2 || splits > 16 || nblk % splits)
    return fail(B2Q_EINVAL, "%s: splits=%d must be 2..16 and divide the %lld blocks of a row", who, splits,
                (long long)nblk);
  if (N > 0 && M > 0 && K > 0 && (ldx < K || (ldx % 4)))
    return fail(B2Q_EALIGN, "%s: ldx must be >= K and a multiple of 4", who);
  const size_t need = (size_t)splits * (size_t)M * (size_t)N * sizeof(float);
  if (need > workspace_bytes)
    return fail(B2Q_ERANGE, "%s: %d splits x M=%lld x N=%lld partial sums need %zu bytes, the scratch holds %zu", who,
                splits, (long long)M, (long long)N, need, workspace_bytes);
  LaunchArgs a{};
  a.fmt = fmt;
  a.wq = wq, a.ldwq = ldwq, a.ws = ws, a.x_f32 = x, a.ldx = ldx, a.y = y, a.ldy = N;
  a.N = N, a.K = K, a.M = M;
  a.workspace = workspace, a.workspace_bytes = workspace_bytes, a.force_splits = splits;
  return launch_gemv(a, stream);
}

}  // namespace b2q

using namespace b2q;

extern "C" {

int b2q_gemv_q4_0(const uint8_t* wq, int64_t ldwq, const int16_t* ws, const int8_t* xq, const float* xd, float* y,
                  int32_t* s, int64_t N, int64_t K, int64_t M, int variant, b2q_stream_t stream) {
  int rc = check_gemv_args("b2q_gemv_q4_0", 0, wq, ldwq, ws, xq, xd, y, N, K, M, false);
  if (rc) return rc;
  if (variant < 0 || variant > 2) return fail(B2Q_EINVAL, "b2q_gemv_q4_0: variant %d not in 0..2", variant);
  if (s && !aligned(s, 4)) return fail(B2Q_EALIGN, "b2q_gemv_q4_0: s must be 4-byte aligned");
  LaunchArgs a{};
  a.fmt = 0;
  a.bytes = variant == B2Q_VARIANT_BYTES;
  a.wq = wq, a.ldwq = ldwq, a.ws = ws, a.xq = xq, a.xd = xd, a.y = y, a.ldy = N, a.s = s;
  a.N = N, a.K = K, a.M = M;
  return launch_gemv(a, (cudaStream_t)stream);
}

int b2q_gemv_tq2_0(const uint8_t* wq, int64_t ldwq, const int16_t* ws, const int8_t* xq, const float* xd, float* y,
                   int32_t* s, int64_t N, int64_t K, int64_t M, int variant, b2q_stream_t stream) {
  int rc = check_gemv_args("b2q_gemv_tq2_0", 1, wq, ldwq, ws, xq, xd, y, N, K, M, false);
  if (rc) return rc;
  if (variant < 0 || variant > 2) return fail(B2Q_EINVAL, "b2q_gemv_tq2_0: variant %d not in 0..2", variant);
  if (s && !aligned(s, 4)) return fail(B2Q_EALIGN, "b2q_gemv_tq2_0: s must be 4-byte aligned");
  LaunchArgs a{};
  a.fmt = 1;
  a.bytes = variant == B2Q_VARIANT_BYTES;
  a.wq = wq, a.ldwq = ldwq, a.ws = ws, a.xq = xq, a.xd = xd, a.y = y, a.ldy = N, a.s = s;
  a.N = N, a.K = K, a.M = M;
  return launch_gemv(a, (cudaStream_t)stream);
}

int b2q_gemv_iq4_nl(const uint8_t* wq, int64_t ldwq, const int16_t* ws, const int8_t* xq, const float* xd, float* y,
                    int32_t* s, int64_t N, int64_t K, int64_t M, int variant, b2q_stream_t stream) {
  int rc = check_gemv_args("b2q_gemv_iq4_nl", 3, wq, ldwq, ws, xq, xd, y, N, K, M, false);
  if (rc) return rc;
  if (variant < 0 || variant > 2) return fail(B2Q_EINVAL, "b2q_gemv_iq4_nl: variant %d not in 0..2", variant);
  if (s && !aligned(s, 4)) return fail(B2Q_EALIGN, "b2q_gemv_iq4_nl: s must be 4-byte aligned");
  LaunchArgs a{};
  a.fmt = 3;
  a.bytes = variant == B2Q_VARIANT_BYTES;
  a.wq = wq, a.ldwq = ldwq, a.ws = ws, a.xq = xq, a.xd = xd, a.y = y, a.ldy = N, a.s = s;
  a.N = N, a.K = K, a.M = M;
  return launch_gemv(a, (cudaStream_t)stream);
}

int b2q_gemv_q4_k(const uint8_t* wq, int64_t ldwq, const int16_t* ws, const int8_t* xq, const float* xd, float* y,
                  int32_t* s, int64_t N, int64_t K, int64_t M, int variant, b2q_stream_t stream) {
  int rc = check_gemv_args("b2q_gemv_q4_k", 4, wq, ldwq, ws, xq, xd, y, N, K, M, false);
  if (rc) return rc;
  if (variant < 0 || variant > 2) return fail(B2Q_EINVAL, "b2q_gemv_q4_k: variant %d not in 0..2", variant);
  if (s && !aligned(s, 4)) return fail(B2Q_EALIGN, "b2q_gemv_q4_k: s must be 4-byte aligned");
  LaunchArgs a{};
  a.fmt = 4;
  a.wq = wq, a.ldwq = ldwq, a.ws = ws, a.xq = xq, a.xd = xd, a.y = y, a.ldy = N, a.s = s;
  a.N = N, a.K = K, a.M = M;
  return launch_gemv(a, (cudaStream_t)stream);
}

int b2q_gemv_q8_0(const uint8_t* wq, int64_t ldwq, const int16_t* ws, const int8_t* xq, const float* xd, float* y,
                  int32_t* s, int64_t N, int64_t K, int64_t M, int variant, b2q_stream_t stream) {
  int rc = check_gemv_args("b2q_gemv_q8_0", 2, wq, ldwq, ws, xq, xd, y, N, K, M, false);
  if (rc) return rc;
  if (variant < 0 || variant > 2) return fail(B2Q_EINVAL, "b2q_gemv_q8_0: variant %d not in 0..2", variant);
  if (s && !aligned(s, 4)) return fail(B2Q_EALIGN, "b2q_gemv_q8_0: s must be 4-byte aligned");
  LaunchArgs a{};
  a.fmt = 2;
  a.bytes = variant == B2Q_VARIANT_BYTES;
  a.wq = wq, a.ldwq = ldwq, a.ws = ws, a.xq = xq, a.xd = xd, a.y = y, a.ldy = N, a.s = s;
  a.N = N, a.K = K, a.M = M;
  return launch_gemv(a, (cudaStream_t)stream);
}

int b2q_quant_gemv(int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws, const float* x, int64_t ldx,
                   int8_t* xq, float* xd, float* y, int64_t N, int64_t K, int64_t M, b2q_stream_t stream) {
  if (!fmt_ok(fmt)) return fail(B2Q_EINVAL, "b2q_quant_gemv: fmt %d is not %s", fmt, fmt_list);
  int rc = check_gemv_args("b2q_quant_gemv", fmt, wq, ldwq, ws, x, nullptr, y, N, K, M, true);
  if (rc) return rc;
  if (N > 0 && M > 0 && K > 0 && (ldx < K || (ldx % 4)))
    return fail(B2Q_EALIGN, "b2q_quant_gemv: ldx must be >= K and a multiple of 4");
  if ((xq == nullptr) != (xd == nullptr)) return fail(B2Q_EINVAL, "b2q_quant_gemv: give both xq and xd, or neither");
  if (xq && !aligned(xq, 16)) return fail(B2Q_EALIGN, "b2q_quant_gemv: xq must be 16-byte aligned");
  if (xd && !aligned(xd, 4)) return fail(B2Q_EALIGN, "b2q_quant_gemv: xd must be 4-byte aligned");
  LaunchArgs a{};
  a.fmt = fmt;
  a.wq = wq, a.ldwq = ldwq, a.ws = ws, a.x_f32 = x, a.ldx = ldx, a.xq_out = xq, a.xd_out = xd, a.y = y, a.ldy = N;
  a.N = N, a.K = K, a.M = M;
  return launch_gemv(a, (cudaStream_t)stream);
}

size_t b2q_workspace_size(int fmt, int64_t N, int64_t K, int64_t M) {
  if (!fmt_ok(fmt) || N <= 0 || K <= 0 || M <= 0 || (K % fmt_block(fmt))) return 0;
  const int tc_min = g_tc_min_m.load();
  if (tc_min > 0 && M >= tc_min && fmt != 3 && fmt != 4) return tc_act_bytes(fmt, N, K, M);  // GEMV ignores it
  // below the threshold, from 2-3 columns at the default one: the tensor-core workspace where the warp-specialized
  // schedule would take this layer (its tiles, K split if need be, fill the GPU), else the GEMV's split-K scratch
  if (tc_min == 8 && M >= ws_min_columns(fmt) && fmt != 3 && fmt != 4 && gemm_tc_ws_bytes(fmt, N, K, M, 1) > 0) {
    DeviceInfo di;
    const int NT = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
    const int64_t tiles = ((N + 127) / 128) * ((M + NT - 1) / NT);
    if (device_info(&di) == B2Q_OK && tiles * gemm_tc_ws_splits(fmt, N, K, M) >= (int64_t)di.sms)
      return tc_act_bytes(fmt, N, K, M);
  }
  const int sp = choose_splits(fmt, K, M);
  return sp > 1 ? (size_t)sp * (size_t)M * (size_t)N * sizeof(float) : 0;
}

int b2q_quant_gemv_ws(int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws, const float* x, int64_t ldx,
                      int8_t* xq, float* xd, float* y, int64_t N, int64_t K, int64_t M, void* workspace,
                      size_t workspace_bytes, b2q_stream_t stream) {
  if (!fmt_ok(fmt)) return fail(B2Q_EINVAL, "b2q_quant_gemv_ws: fmt %d is not %s", fmt, fmt_list);
  int rc = check_gemv_args("b2q_quant_gemv_ws", fmt, wq, ldwq, ws, x, nullptr, y, N, K, M, true);
  if (rc) return rc;
  if (N > 0 && M > 0 && K > 0 && (ldx < K || (ldx % 4)))
    return fail(B2Q_EALIGN, "b2q_quant_gemv_ws: ldx must be >= K and a multiple of 4");
  if ((xq == nullptr) != (xd == nullptr)) return fail(B2Q_EINVAL, "b2q_quant_gemv_ws: give both xq and xd, or neither");
  if (xq && !aligned(xq, 16)) return fail(B2Q_EALIGN, "b2q_quant_gemv_ws: xq must be 16-byte aligned");
  if (workspace && !aligned(workspace, 16)) return fail(B2Q_EALIGN, "b2q_quant_gemv_ws: workspace must be 16-byte aligned");
  LaunchArgs a{};
  a.fmt = fmt;
  a.wq = wq, a.ldwq = ldwq, a.ws = ws, a.x_f32 = x, a.ldx = ldx, a.xq_out = xq, a.xd_out = xd, a.y = y, a.ldy = N;
  a.N = N, a.K = K, a.M = M;
  a.workspace = reinterpret_cast<float*>(workspace), a.workspace_bytes = workspace ? workspace_bytes : 0;
  return launch_gemv(a, (cudaStream_t)stream);
}

int b2q_gemv_allgather(int fmt, const uint8_t* wq, int64_t ldwq, const int16_t* ws, const float* x, int64_t ldx,
                       float* y, void* rx, void* const* rx_peers, int64_t rx_stride, unsigned long long* done,
                       int32_t* status, int64_t row0, int64_t n_local, int64_t N_total, int64_t K, int64_t M,
                       int rank, int nranks, long long spin_limit, b2q_stream_t stream) {
  const char* who = "b2q_gemv_allgather";
  if (!fmt_ok(fmt)) return fail(B2Q_EINVAL, "%s: fmt %d is not %s", who, fmt, fmt_list);
  if (nranks < 1 || rank < 0 || rank >= nranks) return fail(B2Q_EINVAL, "%s: rank %d of %d", who, rank, nranks);
  if (M < 1 || M > kMaxColumns) return fail(B2Q_ERANGE, "%s: M=%lld, 1..%d supported", who, (long long)M, kMaxColumns);
  if (K < 1 || n_local < 1 || row0 < 0 || row0 + n_local > N_total)
    return fail(B2Q_EINVAL, "%s: rows [%lld, %lld) not inside [0, %lld), or K=%lld", who, (long long)row0,
                (long long)(row0 + n_local), (long long)N_total, (long long)K);
  if (!y || !rx || !rx_peers || !done || !status) return fail(B2Q_EINVAL, "%s: null pointer", who);
  if (rx_stride < M * N_total) return fail(B2Q_EINVAL, "%s: rx_stride %lld < M*N_total", who, (long long)rx_stride);
  if (spin_limit < 1) return fail(B2Q_EINVAL, "%s: spin_limit must be positive", who);
  int rc = check_gemv_args(who, fmt, wq, ldwq, ws, x, nullptr, y, n_local, K, M, true);
  if (rc) return rc;
  if (ldx < K || (ldx % 4)) return fail(B2Q_EALIGN, "%s: ldx must be >= K and a multiple of 4", who);
  if (!aligned(rx, 8) || !aligned(done, 8) || !aligned(status, 4))
    return fail(B2Q_EALIGN, "%s: rx/done must be 8-byte aligned, status 4-byte aligned", who);
  LaunchArgs a{};
  a.fmt = fmt;
  a.wq = wq, a.ldwq = ldwq, a.ws = ws, a.x_f32 = x, a.ldx = ldx;
  a.y = y, a.ldy = N_total, a.row0 = row0;
  a.rx = reinterpret_cast<unsigned long long*>(rx), a.rx_peers = reinterpret_cast<unsigned long long* const*>(rx_peers);
  a.rx_stride = rx_stride, a.done = done, a.status = status;
  a.rank = rank, a.nranks = nranks, a.spin_limit = spin_limit;
  a.N = n_local, a.K = K, a.M = M;
  return launch_gemv(a, (cudaStream_t)stream);
}

int b2q_set_tuning(int rows_per_group, int chunks_per_thread, int grid) {
  if (rows_per_group != 0 && rows_per_group != 1 && rows_per_group != 2 && rows_per_group != 4 &&
      rows_per_group != 8 && rows_per_group != 16)
    return fail(B2Q_EINVAL, "b2q_set_tuning: rows_per_group must be 0, 1, 2, 4, 8 or 16");
  if (chunks_per_thread < 0 || grid < 0) return fail(B2Q_EINVAL, "b2q_set_tuning: negative value");
  g_tune_rows = rows_per_group;
  g_tune_cpt = chunks_per_thread;
  g_tune_grid = grid;
  return B2Q_OK;
}

int b2q_set_splitk(int mode) {
  if (mode < 0 || mode > 16) return fail(B2Q_EINVAL, "b2q_set_splitk: mode must be 0 (off), 1 (auto) or 2..16");
  g_splitk_mode = mode;
  return B2Q_OK;
}

int b2q_set_gemm_min_columns(int m) {
  if (m < 0) return fail(B2Q_EINVAL, "b2q_set_gemm_min_columns: m must be >= 0 (0 = never)");
  g_tc_min_m = m;
  return B2Q_OK;
}

int b2q_set_gemm_schedule(int schedule) {
  if (schedule != 0 && schedule != 1)
    return fail(B2Q_EINVAL, "b2q_set_gemm_schedule: 0 (warp-specialized where it applies) or 1 (per-block)");
  g_tc_schedule = schedule;
  return B2Q_OK;
}

int b2q_set_cluster(int ctas) {
  if (ctas != 0 && ctas != 1 && ctas != 2 && ctas != 4 && ctas != 8)
    return fail(B2Q_EINVAL, "b2q_set_cluster: ctas must be 0 (auto), 1 (off), 2, 4 or 8");
  g_tune_cluster = ctas;
  return B2Q_OK;
}

int b2q_set_warps(int warps) {
  if (warps != 0 && (warps < 4 || warps > kMaxThreads / 32))
    return fail(B2Q_EINVAL, "b2q_set_warps: warps must be 0 (auto) or 4..%d", kMaxThreads / 32);
  g_tune_warps = warps;
  return B2Q_OK;
}

int b2q_set_pipeline(int path, int stages) {
  if (path == 3 || path == 4) {  // 3: programmatic dependent launch on, 4: off
    g_pdl = path == 3 ? 1 : 0;
    return B2Q_OK;
  }
  if (path < 0 || path > 5 || path == 3 || path == 4)
    return fail(B2Q_EINVAL, "b2q_set_pipeline: path must be 0 (auto), 1 (ring), 2 (registers), 5 (warp rows)");
  if (stages < 0 || stages == 1 || stages > 8) return fail(B2Q_EINVAL, "b2q_set_pipeline: stages must be 0 or 2..8");
  g_tune_path = path;
  g_tune_stages = stages;
  return B2Q_OK;
}

}  // extern "C"
