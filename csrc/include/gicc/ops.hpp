// ops.hpp -- C++ entry points of the sm_100a kernels (throw std::runtime_error on misuse).
// Every function enqueues on `stream` and returns without synchronising.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "gicc/host_util.hpp"
#include "gicc/types.hpp"

namespace gicc {
namespace ops {

// C[M,N] = alpha * A[M,K] * B[N,K]^T  (bf16 in, f32 accumulate; bf16 or f32 out).
// bn selects the tile: 128 or 256 (one CTA, 128 x bn), 512 (CTA pairs, 256 x 256), 1024 (CTA
// pairs, 256 x 512), 0 = by shape: 1024 when the pair tiles fill the GPU's CTA pairs about as
// evenly as 128 x 256 tiles fill its SMs, else 256.
GICC_EXPORT void gemm_bf16(const void* A, const void* B, void* C, int M, int N, int K, long long lda, long long ldb,
                           long long ldc, bool out_f32, float alpha, int bn, cudaStream_t stream);
// C[M,N] = alpha * A[M,K] * B[N,K]^T on kind::tf32 tensor cores (fp32 words, their tf32 part used);
// bn as gemm_bf16's (256 one CTA, 512 / 1024 CTA pairs, 0 by shape).
GICC_EXPORT void gemm_tf32(const float* A, const float* B, float* C, int M, int N, int K, long long lda, long long ldb,
                           long long ldc, float alpha, cudaStream_t stream, int bn = 0);
// dst[rows][3K]: each src row split into its tf32 part hi and the rest lo = x - hi, laid out
// (hi, hi, lo) for order 0 or (hi, lo, hi) for order 1.
GICC_EXPORT void tf32_split(const float* src, long long ld, int rows, int K, float* dst, int order, cudaStream_t stream);
// fp32 C = alpha * A * B^T on the tensor cores with three tf32 products (Ahi.Bhi + Ahi.Blo +
// Alo.Bhi, one GEMM over 3K); work holds (M + N) * 3K floats.
GICC_EXPORT void gemm_fp32(const float* A, const float* B, float* C, int M, int N, int K, long long lda, long long ldb,
                           long long ldc, float alpha, float* work, cudaStream_t stream, int bn = 0);
// Process-wide tuning of gemm_bf16's 1-CTA kernel (A/B experiments; the defaults are the
// measured configuration): m-blocks per raster group and the L2 eviction hints of the
// operand loads (0 none, 1 keep A / stream B, 2 keep B / stream A).
struct GemmTuning {
  int group_m = 16;       // 1-CTA kernel: 128-row m-blocks per raster group
  int l2_hint = 0;
  int pair_group_m = 16;  // CTA-pair kernels (bn = 512, 1024): 256-row m-blocks per raster group
  int pair_l2_hint = 0;   // CTA-pair kernels: L2 eviction hints as l2_hint
  int pair_prefetch = 0;  // CTA-pair kernels: L2 prefetch of the operands this many k-steps ahead (0 off)
  int pair_tma_store = 1; // CTA-pair kernels: bf16 C stored through shared memory and TMA (1) or per thread (0)
};
GICC_EXPORT void set_gemm_tuning(const GemmTuning& t);
GICC_EXPORT GemmTuning gemm_tuning();
// Self-test of the GEMM core's tile-done ordering: counters must hold 2*tiles+1 zeroed
// words ([warps finished per tile][times published per tile][violations]).
GICC_EXPORT void gemm_tile_done_selftest(const void* A, const void* B, int M, int N, int K, uint32_t* counters,
                                         uint32_t skew_ns, cudaStream_t stream);

// ---- communication kernels (comm.cu) ------------------------------------------------------
GICC_EXPORT void barrier_single(BarrierCtx* ctx, uint64_t* flag, cudaStream_t s);
GICC_EXPORT void barrier_continuous(BarrierCtx* ctx, int n, uint64_t* counter, cudaStream_t s);
// Grid copy of `bytes`, repeated `iters` times, ending with fence.acq_rel.sys (local or peer memory).
// window > bytes: repetition i copies at offset (i*bytes) mod (window-bytes) on both sides.
GICC_EXPORT void copy(void* dst, const void* src, size_t bytes, int iters, int blocks, int threads, cudaStream_t s,
                      size_t window = 0);
// Grid put; each block then adds 1 to *sig_remote with release semantics.
GICC_EXPORT void put_signal(void* dst, const void* src, size_t bytes, uint64_t* sig_remote, int blocks, cudaStream_t s);
GICC_EXPORT void wait_signal(const uint64_t* sig, int cmp, uint64_t value, uint64_t timeout_ns, int* status,
                             cudaStream_t s);
GICC_EXPORT void signal(uint64_t* sig, uint64_t value, int op, cudaStream_t s);
GICC_EXPORT void pingpong(void* remote_buf, const void* local_buf, size_t bytes, uint64_t* remote_flag,
                          const uint64_t* local_flag, int iters, bool initiator, uint64_t base, uint64_t* out_ns,
                          uint64_t timeout_ns, int rank, cudaStream_t s);
GICC_EXPORT void quiet_latency(uint64_t* remote, int iters, uint64_t* out_ns, cudaStream_t s);
GICC_EXPORT void flush_queued(DeviceCtx* ctx, int* status, cudaStream_t s);
GICC_EXPORT void ctx_put(DeviceCtx* ctx, uint64_t laddr, uint32_t lkey, uint64_t raddr, uint32_t rkey, uint32_t size,
                         cudaStream_t s);
GICC_EXPORT void fill_pattern(void* buf, size_t n, uint32_t seed, cudaStream_t s);
// Counts bytes of buf[0, n) that differ from the fill_pattern(seed) bytes at [base, base + n).
GICC_EXPORT void check_pattern(const void* buf, size_t n, uint32_t seed, unsigned long long* bad, cudaStream_t s,
                               size_t base = 0);

// ---- collectives (collectives.cu) ---------------------------------------------------------
enum AllreduceAlgo : int { ALLREDUCE_ONESHOT = 0, ALLREDUCE_TWOSHOT = 1, ALLREDUCE_NVLS = 2 };
// out = scale * sum_i srcs[i] over `count` bf16 elements (f32 accumulation); srcs may be peer memory.
GICC_EXPORT void reduce_bf16(const void* const* srcs, int nsrc, void* out, size_t count, float scale, bool out_f32,
                             cudaStream_t s);
// Allreduce of `count` bf16 elements held in symmetric memory.  in/out: per-rank addresses
// (this process's view); mc_in/mc_out: multicast addresses (NVLS only); flag_bases: per-rank
// base of a [2][max_blocks][n] signal-word area; epoch: call counter (same on all ranks).
// With epoch_dev (a local word, zero before the first call) and ticket (a local 32-bit word,
// zero), the epoch is kept on the device instead: each call uses *epoch_dev + 1 and stores it
// back when its last CTA finishes, so the call can be captured in a CUDA graph and replayed.
GICC_EXPORT void allreduce_bf16(int algo, const void* const* in, void* const* out, const void* mc_in, void* mc_out,
                                int n, int me, size_t count, float scale, bool out_f32, uint64_t* const* flag_bases,
                                int max_blocks, uint64_t epoch, uint64_t timeout_ns, int blocks, cudaStream_t s,
                                uint64_t* epoch_dev = nullptr, unsigned int* ticket = nullptr);

// Reduce-scatter of `count` bf16 elements (count % (8 * n) == 0): rank r receives chunk r of
// the sum (count / n elements, bf16 or f32, scaled) in `out` (local).  nvls: the switch adds
// the copies (mc_in = the input's multicast address); otherwise every rank's input is read
// over NVLink.  Flags, epochs and the device-epoch option as for allreduce_bf16.
GICC_EXPORT void reduce_scatter_bf16(bool nvls, const void* const* in, const void* mc_in, void* out, int n, int me,
                                     size_t count, float scale, bool out_f32, uint64_t* const* flag_bases,
                                     int max_blocks, uint64_t epoch, uint64_t timeout_ns, int blocks, cudaStream_t s,
                                     uint64_t* epoch_dev = nullptr, unsigned int* ticket = nullptr);
// All-gather: this rank's `shard_bytes` (16-byte multiple, local) land at offset
// me * shard_bytes of every rank's symmetric output.  nvls: one multimem store per vector
// (mc_out = the output's multicast address); otherwise one store per rank.
GICC_EXPORT void all_gather(bool nvls, const void* shard, void* const* out, void* mc_out, int n, int me,
                            size_t shard_bytes, uint64_t* const* flag_bases, int max_blocks, uint64_t epoch,
                            uint64_t timeout_ns, int blocks, cudaStream_t s, uint64_t* epoch_dev = nullptr,
                            unsigned int* ticket = nullptr);

// ---- ring-stripe fp32 matmul (ring_mm.cu) -----------------------------------------------------
// One step of C_s = A_s . B over a ring of n ranks: A_s [Ns][N] (my rows), B stripes [N][Ns]
// travelling to the right, C_s [Ns][N].  Counters are monotonic over the whole job: for the
// job's g-th step (g = 0, 1, ...) the host passes arrivals_target = (stripes received so far
// including this one) * push_ctas, consumed_target = steps the right neighbour must have
// finished, ticket_target = (g + 1) * grid.
struct RingMmStep {
  int N = 0, Ns = 0;
  const float* A = nullptr;
  const float* Bcur = nullptr;           // the stripe held this step (own stripe or a landing buffer)
  float* C = nullptr;
  int col_block = 0;                     // the stripe's index: columns [col_block*Ns, +Ns) of C
  float* Bnext_remote = nullptr;         // right neighbour's landing buffer for the next step (null: no push)
  uint64_t* arrivals_remote = nullptr;   // right neighbour's arrival word
  const uint64_t* arrivals = nullptr;    // mine (null: Bcur is local)
  uint64_t arrivals_target = 0;
  const uint64_t* consumed = nullptr;    // mine, advanced by the right neighbour once per finished step
  uint64_t consumed_target = 0;
  uint64_t* consumed_left = nullptr;     // the left neighbour's consumed word (null when alone)
  unsigned long long* ticket = nullptr;  // local count of finished CTAs (monotonic)
  unsigned long long ticket_target = 0;
  int push_ctas = 0;                     // CTAs that forward the stripe (kept for every step)
  // Tensor-core mode (Bsplit non-null): the step kernel's other CTAs write Bcur^T as
  // (hi, lo, hi) tf32 parts into Bsplit [Ns][3N], then a kind::tf32 GEMM with Asplit
  // [Ns][3N] = (hi, hi, lo) of A_s (tf32_split order 0) writes the column block.
  const float* Asplit = nullptr;
  float* Bsplit = nullptr;
  uint64_t timeout_ns = 0;
  int rank = 0, left = -1, right = -1;
};
GICC_EXPORT int ring_mm_grid(int Ns, int push_ctas);
// Grid of a tensor-core-mode step (push CTAs + splitting CTAs).
GICC_EXPORT int ring_mm_grid_tc(int push_ctas);
GICC_EXPORT void ring_mm_step(const RingMmStep& a, cudaStream_t s);

// ---- Jacobi (jacobi.cu) ---------------------------------------------------------------------
struct JacobiStep {
  const float* a = nullptr;  // [rows+2][nx] read buffer
  float* b = nullptr;        // [rows+2][nx] write buffer
  int nx = 0, rows = 0;
  float* top_dst = nullptr;  // upper neighbour's bottom halo row (its write buffer), or null
  float* bot_dst = nullptr;  // lower neighbour's top halo row, or null
  uint64_t* top_sig_remote = nullptr;
  uint64_t* bot_sig_remote = nullptr;
  const uint64_t* top_flag = nullptr;
  const uint64_t* bot_flag = nullptr;
  uint64_t wait_top = 0, wait_bot = 0;
  double* norm = nullptr;
  uint64_t timeout_ns = 0;
  int rank = 0;
};
GICC_EXPORT void jacobi_init(float* a, float* b, int nx, int ny, int rows, int g0, uint64_t seed, cudaStream_t s);
GICC_EXPORT void jacobi_step(const JacobiStep& st, cudaStream_t s);
GICC_EXPORT int jacobi_ctas_per_row(int nx);
// Many iterations in one cooperative launch (per-CTA row blocks, device-side dependencies
// between neighbouring blocks; same halo counters as jacobi_step, so the two can be mixed).
struct JacobiRun {
  float* buf[2] = {nullptr, nullptr};  // [rows+2][nx]; global iteration gi reads buf[gi & 1]
  int nx = 0, rows = 0;
  float* top_dst[2] = {nullptr, nullptr};  // upper neighbour's bottom halo row in its buffer p
  float* bot_dst[2] = {nullptr, nullptr};  // lower neighbour's top halo row in its buffer p
  uint64_t* top_sig_remote = nullptr;
  uint64_t* bot_sig_remote = nullptr;
  const uint64_t* top_flag = nullptr;
  const uint64_t* bot_flag = nullptr;
  uint64_t iter0 = 0;         // global index of the first iteration (iterations done so far)
  int iters = 0;
  uint64_t* done = nullptr;   // [jacobi_persistent_grid(rows)] zeroed once, then monotonic
  double* norm = nullptr;     // optional: sum of squared updates of the last iteration
  uint64_t timeout_ns = 0;
  int rank = 0;
};
GICC_EXPORT int jacobi_persistent_grid(int rows);
GICC_EXPORT void jacobi_run(const JacobiRun& r, cudaStream_t s);

// ---- distributed GEMM with fused NVLink transfers (gemm_dist.cu) ---------------------------
// Pointer arrays are indexed by rank and hold this process's view of each rank's buffer.
struct AgGemmArgs {
  int n = 0, r = 0, M = 0, Ns = 0, K = 0;
  void* a_full[16] = {};       // [M][K] bf16 landing buffers (current parity)
  const void* B = nullptr;     // [Ns][K] bf16 local weights (B^T layout)
  long long ldb = 0;
  void* C = nullptr;           // [M][Ns] bf16 output
  long long ldc = 0;
  uint64_t* arrivals[16] = {}; // [n][M/n/128] arrival counters
  uint64_t* done[16] = {};     // [n] CTA-done counters
  uint64_t epoch = 0;          // call number, >= 1, equal on all ranks
  int units_per_band = 4;
  int grid = 0;
  int comm_ctas = 0;           // CTAs that push the shard (0 = all)
  void* a_mc = nullptr;              // NVLS: multicast view of the landing buffer (current parity)
  uint64_t* arrivals_mc = nullptr;   // NVLS: multicast view of the arrival counters
  uint64_t* tile_counter = nullptr;  // local word, zero before the first call; calls that share
                                     // it must use the same shape and grid (dynamic tile order)
  uint64_t timeout_ns = 0;
  uint64_t* trace = nullptr;   // diagnostics: %globaltimer stamps per tile / unit / CTA
  int diag = 0;                // bit 0 = no transfer (diagnostics: times the math alone);
                               // bit 1 = external transfer (ag_transfer_ce): no pushes, waits kept
  int pair = 0;                // tensor-core tiles: 0 = one CTA, 128 x 256; 1 = CTA pairs, 256 x 256;
                               // 2 = CTA pairs, 256 x 512 (pairs need M/n % 256 == 0, no trace)
};
struct GemmRsArgs {
  int n = 0, r = 0, M = 0, N = 0, K = 0;  // K = local K
  const void* A = nullptr;     // [M][K] bf16 (K-shard)
  long long lda = 0;
  const void* B = nullptr;     // [N][K] bf16 (K-shard, B^T layout)
  long long ldb = 0;
  void* slots[16] = {};        // [n][M/n][N] bf16 partial landing areas (current parity)
  uint64_t* arrivals[16] = {}; // [n][M/n/128]
  uint64_t* done[16] = {};     // [n]
  void* out = nullptr;         // [M/n][N] bf16
  long long ldo = 0;
  uint64_t epoch = 0;
  int grid = 0;
  uint64_t timeout_ns = 0;
  // NVLS mode (staging_mc non-null): slots[r] is this rank's [M][N] bf16 staging buffer
  // (current parity), staging_mc its multicast view; arrivals[o] = owner o's [M/n/128]
  // counters; band_tiles = local [n][M/n/128] words; tile_counter as for ag_gemm.
  const void* staging_mc = nullptr;
  uint64_t* band_tiles = nullptr;
  uint64_t* tile_counter = nullptr;
  int comm_ctas = 0;           // CTAs running the reduce warps (0 = 16)
  int units_per_band = 4;      // row slices per 128-row band (divides 128)
  uint64_t* trace = nullptr;   // NVLS mode diagnostics: %globaltimer stamps (layout at RsNvSched)
  int join_reduce = 0;         // NVLS: CTAs that finished their GEMM tiles join the reduction
  uint64_t* unit_counter = nullptr;  // NVLS + join_reduce: local word, zero before the first call
  int raster_group = 0;        // NVLS: m-blocks per raster group (0 = 16).  Smaller groups finish
                               // bands sooner (the owners can reduce them earlier); larger
                               // ones reuse B better in L2 when B does not fit there
  int pair = 0;                // NVLS: 0 = one CTA per 128 x 256 tile; 1 / 2 = CTA pairs with
                               // 256 x 256 / 256 x 512 tiles (M/n % 256 == 0; no join, no trace)
};
// Memory-model litmus tests (gicc/proto/litmus.hpp).  test 0 = MP (role 0 writes data and
// flag into role 1's memory; role 1 checks), test 1 = SB (each role stores into the other's
// word array, optionally fence.sc, then loads its own copy of the other's word).
struct LitmusRole {
  uint64_t* data = nullptr;          // MP: the reader's data ring (k words)
  uint64_t* flag = nullptr;          // MP: the reader's flag word
  uint64_t* ready_remote = nullptr;  // SB: the other role's ready word
  const uint64_t* ready_local = nullptr;
  uint64_t* mine_remote = nullptr;   // SB: the other role's copy of this role's word array
  const uint64_t* theirs_local = nullptr;
  uint64_t* out = nullptr;           // SB: [iters] loaded values
  uint64_t* result = nullptr;        // [2]: status, MP violations (device memory)
};
struct LitmusArgs {
  int test = 0, iters = 0, k = 64, use_fence = 1;
  uint32_t seed = 1, max_delay = 256;
  uint64_t timeout_ns = 0;
  int role_base = 0;                 // first role run on this GPU
  LitmusRole role[2];
};
GICC_EXPORT void litmus(const LitmusArgs& a, int nroles_here, cudaStream_t s);
// Measurement kernels of the reference's example programs (csrc/kernels/examples.cu).
// phase_loop: one block; stamps = [iters][6] %globaltimer values; bar is advanced by
// 3 * iters epochs (the caller tells the host Barrier with advance()).
GICC_EXPORT void phase_loop(BarrierCtx* bar, float* x, float* y, const float* recv, float* send_remote, size_t n,
                            int iters, float a, int rank, int left, uint64_t* stamps, unsigned long long* bad,
                            cudaStream_t s);
// y = a*x + y and the result stored into dst_remote, per CTA; each CTA adds 1 to
// *arrivals_remote when its chunk is visible.
GICC_EXPORT void saxpy_put(const float* x, float* y, float a, size_t n, float* dst_remote, uint64_t* arrivals_remote,
                           int blocks, cudaStream_t s);
GICC_EXPORT void wait_count(const uint64_t* counter, uint64_t target, uint64_t timeout_ns, int rank, cudaStream_t s);
GICC_EXPORT void saxpy(const float* x, float* y, float a, size_t n, cudaStream_t s);
// `tiles` CTAs each put one pattern tile from shared memory with the bulk tile put
// (device put_tile) to dst + i * tile_bytes (dst may be a peer's memory), then add 1 to sig.
GICC_EXPORT void put_tile_test(void* dst, int tiles, uint32_t tile_bytes, uint32_t seed, uint64_t* sig,
                               cudaStream_t s);
// Copy-engine transfer for ag_gemm (the A/B alternative to SM pushes): on stream `s`, for
// each peer d in the consumption order (r-1, r-2, ...): wait (stream memory operation)
// until d finished the call that last used this parity, copy this rank's shard into d's
// landing buffer with cudaMemcpyAsync, `chunks` pieces per peer, and after each piece write
// d's arrival counters of its bands to epoch * units_per_band.  No SM issues NVLink
// traffic; launch ag_gemm with diag bit 1 (external transfer) on another stream.
// The peer-progress wait is a one-thread kernel on `s` bounded by timeout_ns (0 = the
// configured default); on timeout it records GICC_ETIMEDOUT and the copies go ahead.
struct AgCeArgs {
  int n = 0, r = 0, M = 0, K = 0;
  void* a_full[16] = {};        // each rank's landing buffer (current parity), mapped here
  uint64_t* arrivals[16] = {};  // each rank's [n][M/n/128] counters, mapped here
  const uint64_t* done_local = nullptr;  // [n] CTA-exit counts received from each rank
  uint64_t epoch = 0;
  int grid = 0;                 // CTAs of the ag_gemm launch (done-counter unit)
  int units_per_band = 4;
  int chunks = 4;               // copies per peer (each followed by its bands' counters)
  uint64_t timeout_ns = 0;      // bound of the peer-progress wait (0 = default)
};
GICC_EXPORT void ag_transfer_ce(const AgCeArgs& a, cudaStream_t s);
GICC_EXPORT void ag_gemm(const AgGemmArgs& a, cudaStream_t s);
GICC_EXPORT void gemm_rs(const GemmRsArgs& a, cudaStream_t s);

// ---- MoE expert-parallel layer (moe.cu) -----------------------------------------------------
struct MoeWorkspace {          // local device arrays
  int* dest_row_base = nullptr;  // [E]
  int* key_base = nullptr;       // [El*n + 1]
  int* key_cursor = nullptr;     // [El*n]
  int* expert_base = nullptr;    // [El]
  int* expert_rows = nullptr;    // [El]
  int* mblk_prefix = nullptr;    // [El+1]
  uint64_t* cum_rows = nullptr;  // [n][El], zero-initialised once
  uint64_t* cum_pairs = nullptr; // [1], zero-initialised once
  int* send_pair = nullptr;      // [T*topk]
  int* send_row = nullptr;       // [T*topk]
  uint64_t* g1_tile_ctr = nullptr; // [2], zero-initialised once (needed with dispatch_ctas)
  uint64_t* g2_ctr = nullptr;      // [6], zero-initialised once (needed with combine_ctas)
  uint64_t* g2_queue = nullptr;    // [cap/128 * H/256] (needed with combine_ctas)
};
struct MoeArgs {
  int n = 1, r = 0, T = 0, H = 0, I = 0, E = 0, topk = 8;
  const float* logits = nullptr;  // [T][E] router logits
  const void* x = nullptr;        // [T][H] bf16 tokens
  const void* w1 = nullptr;       // [El][2I][H] bf16, rows interleaved per 128: gate blk, up blk
  const void* w2 = nullptr;       // [El][H][I] bf16
  int* topk_idx = nullptr;        // [T*topk]
  float* topk_w = nullptr;        // [T*topk]
  int* counts = nullptr;          // [E]
  void* count_tab[8] = {};        // per rank: [n][E] int32 (parity of this call)
  uint64_t* plan_flags[8] = {};   // per rank: [n] words
  void* recv[8] = {};             // per rank: [cap][H] bf16 (parity of this call)
  void* meta[8] = {};             // per rank: [cap] int4 (parity of this call)
  uint64_t* arrivals[8] = {};     // per rank: [n][El] words
  void* h = nullptr;              // [cap][I] bf16 local
  void* comb[8] = {};             // per rank: [T*topk][H] bf16
  uint64_t* comb_arrivals[8] = {};// per rank: [1] word
  void* out = nullptr;            // [T][H] bf16
  int cap_rows = 0;
  uint64_t epoch = 0;             // call number >= 1
  uint64_t timeout_ns = 0;
  MoeWorkspace ws;
  float* stage_ms = nullptr;      // optional host [6]: per-stage device time (synchronises)
  int dispatch_ctas = 0;          // CTAs whose warps dispatch (0 = every CTA); with fewer, the
                                  // first GEMM takes tiles dynamically (ws.g1_tile_ctr)
  int combine_ctas = 0;           // > 0: the second GEMM stages its rows in y_stage and only this
                                  // many CTAs push them to the sources (ws.g2_ctr, ws.g2_queue)
  void* y_stage = nullptr;        // [cap][H] bf16 local (needed with combine_ctas)
  int comm_only = 0;              // 1: identity experts -- route, dispatch, return, combine only
                                  // (out[t] = sum_j w_j * x[t]), to time the all-to-all round trip
};
GICC_EXPORT void moe_route(const float* logits, int T, int E, int topk, int* topk_idx, float* topk_w, int* counts,
                           cudaStream_t s);
GICC_EXPORT void moe_forward(const MoeArgs& a, cudaStream_t s);

}  // namespace ops
}  // namespace gicc
