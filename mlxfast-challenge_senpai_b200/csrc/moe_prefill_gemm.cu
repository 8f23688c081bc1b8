// Prefill MoE expert block: expert-sorted grouped GEMMs on the 5th-generation
// tensor cores (tcgen05), weights dequantized into TMEM.
//
// Rows are the (token, slot) pairs in expert order (b2_moe_gather_sort); an
// expert's rows are cut into token tiles of at most NMAX rows (balanced
// split, N = rows rounded up to 16).  A work unit is (token tile, block of
// 128 weight rows); every CTA walks the units u = cta, cta + G, ... and per
// unit streams the K range in stages of 128:
//   weights [128 x 128]: one 9 KB bulk copy of packed NVFP4 codes and scale
//     bytes from the prefill bank (b2_moe_prepare_prefill_bank), dequantized
//     exactly to bf16 (hardware E2M1 -> f16, a shift, one bf16 multiply by
//     the scale) by eight warps straight into TMEM with tcgen05.st: the A operand
//     comes from tensor memory and never touches shared memory;
//   tokens [N x 128] bf16: two tiled TMA copies (box N x 64, 128-byte
//     swizzle) of the rows of the tile -- gate/up: the token rows gathered
//     into expert order; down: the SwiGLU rows;
//   one thread issues 8 MMAs of 128 x N x 16 (A from TMEM, B from shared
//   memory) into a TMEM accumulator; two accumulators of NMAX columns
//   alternate between units so the epilogue of one unit overlaps the next.
// Measured on B200: a single thread issues one tcgen05.mma in ~50 cycles,
// the tensor pipe queues about four MMAs, and every barrier wait, fence or
// commit that follows MMAs in the issuing warp waits until they have been
// handed to the pipe, so two warps issue alternate stages (one handshakes
// while the other issues); the per-stage copies come from four
// producer warps taking stages in turn (one issuing thread caps the copy
// rate well below what the MMAs consume).
// Epilogues: the four epilogue warps round their TMEM rows to bf16 into
// shared memory (80 token columns per pass) and release the accumulator,
// then all 128 threads write 16-byte chunks: gate/up -- the 128 weight rows
// are 64 gate rows and the same 64 up rows, act[row] = the reference's bf16
// SwiGLU steps (SiLU from an exact shared-memory table for |g| in
// [2^-8, 2^8), the exact chain otherwise); down -- the 128 hidden outputs
// into y[row] (the per-slot expert output; the ordered weighted combine
// follows in b2_moe_combine).
//
// Warp roles (24 warps): 0 and 5 MMA issue on alternate stages (0 also
// allocates TMEM), 1-4 producers, 8-11 and 20-23 epilogue (two sets taking
// alternate 32-column passes, TMEM lane quarter = warp % 4), 12-19
// dequantizers (two groups of four, each taking one K half of every stage,
// lane quarter = warp % 4).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "moe.cuh"
#include "moe_prefill_gemm.cuh"

namespace b2 {
namespace pf {
namespace {

constexpr int BK = 128;                   // K per stage
constexpr int MW = 128;                   // weight rows per unit (TMEM lanes)
constexpr int NMAX = 160;                 // token rows per tile
constexpr int kMaps = NMAX / 16;          // one tensor map per tile height 16, 32, ..., NMAX
constexpr int S = 4;                      // shared-memory stages (tokens + packed weights)
constexpr int SA = 3;                     // TMEM weight slots
constexpr int SUB_BYTES = NMAX * 64 * 2;  // one 64-wide token sub-tile (20 KB)
constexpr int TOK_BYTES = 2 * SUB_BYTES;
constexpr int W_BYTES = MW * BK / 2 + MW * BK / 16;  // 9216: codes [4][128][16 B], scales [128][8]
constexpr int STAGE_BYTES = (TOK_BYTES + W_BYTES + 1023) / 1024 * 1024;
constexpr int XCH_OFF = S * STAGE_BYTES;  // epilogue staging, per set: bf16 [32 columns][128 rows]
constexpr int XCH_COLS = 32;
constexpr int XCH_BYTES = XCH_COLS * MW * 2;  // per epilogue set
// SiLU of the bf16 values with |g| in [2^-8, 2^8) (exponent fields 119..134,
// both signs): 4096 entries; other values take the exact chain in registers
constexpr int STAB_OFF = XCH_OFF + 2 * XCH_BYTES;
constexpr int STAB_BYTES = 4096 * 2;
constexpr int SROW_OFF = STAB_OFF + STAB_BYTES;  // down: [NMAX] output rows of the tile
// Pair mode (2-CTA tcgen05, cta_group::2; opt-in, B2_PREFILL_PAIR=1): the
// two CTAs of a cluster share one token tile -- each loads half of its rows,
// the MMA reads both halves -- and each holds its own 128-row weight block
// (M = 256 per MMA), so a CTA's shared-memory traffic per stage is ~29 KB
// instead of ~49 KB for the same MMA work; six stages fit.  The odd CTA's
// dequantizer and epilogue warps arrive on their own barriers and one of
// its idle MMA warps forwards each completed phase to the even CTA's.
template <bool PAIR>
struct Geo {
  static constexpr int S = PAIR ? 6 : 4;                    // shared-memory stages
  static constexpr int ROWS = PAIR ? NMAX / 2 : NMAX;       // token rows per CTA and stage
  static constexpr int SUB = ROWS * 64 * 2;                 // one 64-wide token sub-tile
  static constexpr int TOK = 2 * SUB;
  static constexpr int STAGE = (TOK + W_BYTES + 1023) / 1024 * 1024;
  static constexpr int XCH = S * STAGE;
  static constexpr int STAB = XCH + 2 * XCH_BYTES;
  static constexpr int SROW = STAB + STAB_BYTES;
  static constexpr int SMEM = SROW + NMAX * 4 + 1024;
  static_assert(SUB % 1024 == 0 && STAGE % 1024 == 0, "swizzle atoms stay 1024-byte aligned");
  static_assert(SMEM <= 232448, "shared memory per block");
};
constexpr int kMaxS = 6;
constexpr int kWarps = 24;
constexpr int kThreads = kWarps * 32;
constexpr int W_MMA = 0, W_MMA2 = 5, W_PROD = 1, N_PROD = 4, W_EPI = 8, W_EPI2 = 20, W_DQ = 12;
constexpr int kHandoffBar = 2;  // named barrier: the two MMA warps hand stages over, once per stage
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kACol = 2 * NMAX;  // weight slots (64 columns each) follow the two accumulators
static_assert(kACol + SA * 64 <= kTmemCols, "TMEM budget");
static_assert(SUB_BYTES % 1024 == 0 && STAGE_BYTES % 1024 == 0, "swizzle atoms stay 1024-byte aligned");
static_assert(W_EPI % 4 == 0 && W_EPI2 % 4 == 0 && W_DQ % 4 == 0, "lane quarter = warp % 4");
constexpr uint32_t kWaitLimit = 1u << 22;
// kind::f16, both operands K-major, f32 accumulate, M = 128; N is added per
// unit.  Gate/up (mode 0): f16 A and B (format 0); down (mode 1): bf16 A
// and B (format 1).
constexpr uint32_t kIdescF16 = (1u << 4) | ((uint32_t)(MW >> 4) << 24);
constexpr uint32_t kIdescBF16 = kIdescF16 | (1u << 7) | (1u << 10);
// pair mode: M = 256 (128 rows in each CTA's TMEM)
constexpr uint32_t kIdescM256 = (uint32_t)((2 * MW) >> 4) << 24;
constexpr uint32_t kIdescMMask = 0x1fu << 24;

struct Params {
  const uint8_t* wbank;  // this mode's bank: [E][MT][KS][W_BYTES]
  const int4* tiles;     // (first sorted row, rows, expert, N)
  const int* ntiles;
  uint16_t* out;             // gate/up: act [rows][F] (sorted rows); down: y [rows][H] (order[row] if given)
  const uint16_t* silu_tab;  // exact bf16 SiLU table or null
  const uint32_t* order;     // down: sorted row -> (token, slot) row of the output, or null
  // down, expert parallel: output row r lives on rank r / peer_rows at local
  // row r % peer_rows of that rank's buffer peer_out[rank] (peer memory
  // mapped into this process); null for a local output
  uint16_t* const* peer_out;
  uint32_t peer_rows;
  const int* tok_exp;        // gate/up: per sorted row, the f16 pre-scale exponent p of its token
  unsigned* status;
  int MT, KS, ldo;  // weight blocks per tile, K stages, output row length
};

struct TokMaps {
  CUtensorMap m[kMaps];  // box 64 x 16(i+1)
};

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  // K-major operand, 128-byte swizzle: start >> 4, LBO 16 B, SBO 1024 B (one
  // 8-row swizzle atom), descriptor version 1, layout type 2 (SWIZZLE_128B)
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Bounded mbarrier wait that gives up for good once any wait in the CTA has
// timed out (so a broken pipeline ends instead of stacking timeouts).
__device__ __forceinline__ void wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort_flag, unsigned* status) {
  if (*abort_flag) return;
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return;
    if ((i & 255u) == 255u && *abort_flag) return;
  }
  *abort_flag = 1;
  report_status(status, B2_STATUS_WAIT_TIMEOUT);
}

// wait_bar with acquire at cluster scope (pair mode: barriers that receive
// the other CTA's arrivals or the pair's multicast commits).
__device__ __forceinline__ void wait_bar_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                 unsigned* status) {
  if (*abort_flag) return;
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return;
    if ((i & 255u) == 255u && *abort_flag) return;
  }
  *abort_flag = 1;
  report_status(status, B2_STATUS_WAIT_TIMEOUT);
}
template <bool PAIR>
__device__ __forceinline__ void wait_any(uint64_t* bar, uint32_t parity, volatile int* abort_flag, unsigned* status) {
  if (PAIR)
    wait_bar_cluster(bar, parity, abort_flag, status);
  else
    wait_bar(bar, parity, abort_flag, status);
}

// Spinning variant (mbarrier.test_wait never suspends the thread, so the
// waiter resumes as soon as the phase completes) for the MMA-issuing warps.
__device__ __forceinline__ void spin_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, unsigned* status) {
  if (*abort_flag) return;
  for (uint32_t i = 0; i < (kWaitLimit << 4); ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return;
    if ((i & 1023u) == 1023u && *abort_flag) return;
  }
  *abort_flag = 1;
  report_status(status, B2_STATUS_WAIT_TIMEOUT);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Half a 128-wide K stage: 4 MMAs of 128 x N x 16, A (weights) from TMEM
// columns a .. a+31 (8 per MMA), B (tokens) from the swizzled 64-wide
// sub-tile at descriptor b (+32 bytes = +2 per MMA); the first MMA
// overwrites D unless `acc`.
__device__ __forceinline__ void mma_half(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p0, p1;\n\t"
      "setp.ne.b32 p0, %4, 0;\n\t"
      "setp.eq.b32 p1, %4, %4;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%5], %6, %3, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%7], %8, %3, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%9], %10, %3, p1;\n\t}\n" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc), "r"(a + 8), "l"(b + 2), "r"(a + 16), "l"(b + 4), "r"(a + 24), "l"(b + 6)
      : "memory");
}

// mma_half for the 2-CTA pair (issued by the even CTA of the cluster): D and
// A at the same TMEM addresses in both CTAs (each holds its 128 weight rows),
// B = the two CTAs' token halves at the same shared-memory offset.
__device__ __forceinline__ void mma_half_pair(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p0, p1;\n\t"
      "setp.ne.b32 p0, %4, 0;\n\t"
      "setp.eq.b32 p1, %4, %4;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%5], %6, %3, p1;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%7], %8, %3, p1;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%9], %10, %3, p1;\n\t}\n" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc), "r"(a + 8), "l"(b + 2), "r"(a + 16), "l"(b + 4), "r"(a + 24), "l"(b + 6)
      : "memory");
}
// Commit of the pair's MMAs, arriving on the barrier at this offset in both
// CTAs of the cluster.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on the barrier at this offset in CTA 0 of the cluster, relaxed (a
// release at cluster scope blocks the arriving thread ~1,800 cycles).  Used
// only to forward a local barrier phase: the eight warps that completed it
// had waited for their TMEM stores to finish (tcgen05.wait::st) and fenced
// them (tcgen05.fence::before_thread_sync) before their release arrivals,
// and this thread observed that phase (acquire) before forwarding it, so
// the stores are complete before the arrival is issued; the waiting MMA
// thread orders its MMAs after the wait with tcgen05.fence::after_thread_sync.
__device__ __forceinline__ void arrive_leader(uint64_t* bar) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(remote) : "r"(smem_u32(bar)));
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}
// Spinning wait with acquire at cluster scope (barriers that receive arrivals
// from the other CTA of the pair).
__device__ __forceinline__ void spin_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                  unsigned* status) {
  if (*abort_flag) return;
  for (uint32_t i = 0; i < (kWaitLimit << 4); ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return;
    if ((i & 1023u) == 1023u && *abort_flag) return;
  }
  *abort_flag = 1;
  report_status(status, B2_STATUS_WAIT_TIMEOUT);
}

// 32 consecutive TMEM columns of this thread's lane (warp-wide store).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Exact NVFP4 -> bf16 with one conversion instruction per pair: the hardware
// E2M1 -> f16 conversion gives f16 bits (e << 10 | m << 9) of the value v;
// shifted right by 3 (sign kept in place) they are the bf16 bits of
// v * 2^-112 (bf16 exponent field = the f16 biased exponent, bias 127 vs 15;
// zero stays zero); one bf16 multiply by |scale| * 2^112 then gives v * scale
// exactly (at most 6 significant bits, no rounding).
__device__ __forceinline__ uint32_t e2m1x2_to_bf16x2_scaled(uint32_t c16, uint32_t s2) {
  const uint32_t x = ((c16 & 0x7fff7fffu) >> 3) | (c16 & 0x80008000u);
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(x), "r"(s2));
  return d;
}

// bf16x2 (both halves) of |scale| * 2^112 from a prepared scale byte pb (the
// f16 bits of |scale| >> 7, a normal f16 or zero): bf16 bits of |scale| are
// (pb << 4) + (112 << 7); times 2^112 adds another 112 to the exponent.
__device__ __forceinline__ uint32_t bf16_scale2(uint32_t pb) {
  const uint32_t b = pb ? (pb << 4) + 0x7000u : 0u;
  return b * 0x00010001u;
}

// 8 codes of word w (elements 8i..8i+7 of a K group) times the scale s2 ->
// 4 bf16x2 TMEM columns.
__device__ __forceinline__ void dq_word(uint32_t w, uint32_t s2, uint32_t* o) {
  o[0] = e2m1x2_to_bf16x2_scaled(cvt_byte<0>(w), s2);
  o[1] = e2m1x2_to_bf16x2_scaled(cvt_byte<1>(w), s2);
  o[2] = e2m1x2_to_bf16x2_scaled(cvt_byte<2>(w), s2);
  o[3] = e2m1x2_to_bf16x2_scaled(cvt_byte<3>(w), s2);
}

// f16x2 (both halves) of |scale| from a prepared scale byte pb (the f16 bits
// of |scale| >> 7).
__device__ __forceinline__ uint32_t f16_scale2(uint32_t pb) { return (pb << 7) * 0x00010001u; }

// 8 codes of word w times the f16 scale s2 -> 4 f16x2 TMEM columns
// (E2M1 x E4M3 scale has at most 6 significant bits and lies inside the f16
// normal range: exact).
__device__ __forceinline__ void dq_word_f16(uint32_t w, uint32_t s2, uint32_t* o) {
  o[0] = hmul2_u32(cvt_byte<0>(w), s2);
  o[1] = hmul2_u32(cvt_byte<1>(w), s2);
  o[2] = hmul2_u32(cvt_byte<2>(w), s2);
  o[3] = hmul2_u32(cvt_byte<3>(w), s2);
}

// Position of bf16 bits b in the shared SiLU window, or -1 outside it.
__device__ __forceinline__ int silu_window_index(uint32_t b) {
  const uint32_t e = ((b >> 7) & 0xffu) - 119u;
  return e < 16u ? (int)(((b >> 15) << 11) | (e << 7) | (b & 127u)) : -1;
}
__device__ __forceinline__ uint32_t silu_window_bits(int i) {
  return ((uint32_t)(i >> 11) << 15) | ((uint32_t)(119 + ((i >> 7) & 15)) << 7) | (uint32_t)(i & 127);
}
__device__ __forceinline__ uint32_t silu_lookup_bits(const uint16_t* stab, uint32_t gb) {
  const int i = silu_window_index(gb);
  return i >= 0 ? (uint32_t)stab[i] : (uint32_t)f32_to_bf16_bits(silu_bf16(bf16_bits_to_f32((uint16_t)gb)));
}
// bf16x2 multiply: the exact product of two bf16 values (at most 16
// significant bits) rounded once to bf16 -- the reference's
// bf16(silu(g) * u) step for two features at a time.
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// f32 pair -> bf16x2 (round to nearest even; one instruction).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&b);
}

__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

template <int MODE, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1) expert_gemm_kernel(Params p, const __grid_constant__ TokMaps maps) {
  using Gm = Geo<PAIR>;
  constexpr int S = Gm::S;
  constexpr int STAGE_BYTES = Gm::STAGE, SUB_BYTES = Gm::SUB, TOK_BYTES = Gm::TOK;
  constexpr int XCH_OFF = Gm::XCH, STAB_OFF = Gm::STAB, SROW_OFF = Gm::SROW;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[kMaxS], empty[kMaxS], afull[SA], aempty[SA], tfull[2], tempty[2], drain;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // pair mode: the cluster's two CTAs walk the same units; rank rk holds
  // weight block 2 * (unit block) + rk and token rows [rk * N/2, (rk+1) * N/2)
  const int rk = PAIR ? (int)cluster_ctarank() : 0;
  const int G = PAIR ? (int)gridDim.x / 2 : (int)gridDim.x;
  const int cta = PAIR ? (int)blockIdx.x / 2 : (int)blockIdx.x;
  uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);

  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < SA; ++i) {
      // all eight dequantizer warps; pair mode: the even CTA's also counts the
      // one arrival relayed for the odd CTA's eight
      mbar_init(&afull[i], PAIR && rk == 0 ? 9 : 8);
      mbar_init(&aempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 2);  // one commit from each MMA warp
      mbar_init(&tempty[i], PAIR && rk == 0 ? 9 : 8);  // every epilogue warp of both sets (+ the relay)
    }
    mbar_init(&drain, 2);
    fence_mbar_init();
    s_abort = 0;
  }
  if (MODE == 0) {
    uint16_t* stab = reinterpret_cast<uint16_t*>(base + STAB_OFF);
    for (int i = tid; i < 4096; i += kThreads) {
      const uint32_t b = silu_window_bits(i);
      stab[i] = p.silu_tab ? p.silu_tab[b] : f32_to_bf16_bits(silu_bf16(bf16_bits_to_f32((uint16_t)b)));
    }
  }
  if (warp == W_MMA) {
    if (PAIR) {
      // the same warp of both CTAs allocates (the same columns in each)
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                   "r"(kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                   "r"(kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  // pair mode: both CTAs' barriers are initialised before either CTA
  // arrives on, or commits to, the other's
  if (PAIR) cluster_sync_all();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s_tmem;
  volatile int* abort_flag = &s_abort;
  const int MT = p.MT, KS = p.KS;
  const int MTU = PAIR ? MT / 2 : MT;  // units per tile
  const int U = *p.ntiles * MTU;

  if ((warp == W_MMA || warp == W_MMA2) && (!PAIR || rk == 0)) {
    // (pair mode: the even CTA issues the pair's MMAs and commits them to
    // both CTAs' barriers; the odd CTA's MMA warps idle)
    // Two MMA-issuing warps take alternate stages.  Any barrier wait, fence
    // or commit that follows MMAs in the issuing warp stalls until those MMAs
    // have been handed to the tensor pipe, so a single issuing warp leaves the
    // pipe idle during its per-stage handshakes; with two warps, one waits
    // for its next stage and commits while the other issues.  A stage goes:
    // wait for its weight slot (the dequantizers release it only after the
    // stage's copies landed, so afull alone says both operands are in place;
    // on a unit's first stage also for the accumulator), take over from the
    // other warp (rendezvous), 8 MMAs, hand over, commit the stage's smem
    // and TMEM slots.  The tcgen05 fences around the rendezvous order the
    // two warps' MMAs on the shared accumulator.  Both warps commit the
    // unit's tfull barrier (count 2), so it fires when all of the unit's MMAs
    // have completed whichever warp issued them.
    const int mw = warp == W_MMA ? 0 : 1;
    const uint64_t tdesc0 = sw128_desc(smem_u32(base));
    const int my_units = cta < U ? (U - cta + G - 1) / G : 0;
    const uint32_t gend = (uint32_t)my_units * (uint32_t)KS;
    uint32_t g = 0;
    int i = 0;
    for (int u = cta; u < U; u += G, ++i) {
      const int4 tl = p.tiles[u / MTU];
      uint32_t idesc = (MODE == 0 ? kIdescF16 : kIdescBF16) | ((uint32_t)(tl.w >> 3) << 17);
      if (PAIR) idesc = (idesc & ~kIdescMMask) | kIdescM256;
      const int acc = i & 1;
      const uint32_t d = tmem + (uint32_t)(acc * NMAX);
      const bool live = !*abort_flag;  // once per unit: no more MMAs after a timeout
      for (int s = 0; s < KS; ++s, ++g) {
        if ((int)(g & 1u) != mw) continue;
        const uint32_t sl = g % S, as = g % SA;
        if (lane == 0) {
          if (PAIR) {
            if (s == 0) spin_wait_cluster(&tempty[acc], (uint32_t)(((i >> 1) & 1) ^ 1), abort_flag, p.status);
            spin_wait_cluster(&afull[as], (g / SA) & 1u, abort_flag, p.status);
          } else {
            if (s == 0) spin_wait(&tempty[acc], (uint32_t)(((i >> 1) & 1) ^ 1), abort_flag, p.status);
            spin_wait(&afull[as], (g / SA) & 1u, abort_flag, p.status);
          }
        }
        __syncwarp();
        if (g > 0) named_sync(kHandoffBar, 64);  // the other warp has issued stage g - 1
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (lane == 0 && live) {
          const uint64_t b0 = tdesc0 + (uint64_t)(sl * (STAGE_BYTES >> 4));
          const uint32_t a = tmem + kACol + as * 64;
          if (PAIR) {
            mma_half_pair(d, a, b0, idesc, s > 0 ? 1u : 0u);
            mma_half_pair(d, a + 32, b0 + (SUB_BYTES >> 4), idesc, 1u);
          } else {
            mma_half(d, a, b0, idesc, s > 0 ? 1u : 0u);
            mma_half(d, a + 32, b0 + (SUB_BYTES >> 4), idesc, 1u);
          }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (g + 1 < gend) named_sync(kHandoffBar, 64);  // stage g issued
        if (lane == 0) {
          if (PAIR) {
            mma_commit_pair(&empty[sl]);
            mma_commit_pair(&aempty[as]);
          } else {
            mma_commit(&empty[sl]);
            mma_commit(&aempty[as]);
          }
        }
      }
      if (lane == 0) {
        if (PAIR)
          mma_commit_pair(&tfull[acc]);
        else
          mma_commit(&tfull[acc]);
      }
    }
    if (lane == 0) {
      // every MMA of this CTA (both warps) has completed before TMEM is released
      if (PAIR)
        mma_commit_pair(&drain);
      else
        mma_commit(&drain);
      if (mw == 0 && !mbar_wait_bounded(&drain, 0, p.status, kWaitLimit)) *abort_flag = 1;
    }
  } else if (warp >= W_PROD && warp < W_PROD + N_PROD) {
    if (lane == 0) {
      const int pi = warp - W_PROD;
      const int my_units = cta < U ? (U - cta + G - 1) / G : 0;
      const uint32_t gend = (uint32_t)my_units * (uint32_t)KS;
      const uint32_t gtail = gend > (uint32_t)S ? gend - S : 0u;
      uint32_t tail_issued = 0;  // bit (g - gtail) for the last S stages this warp issued
      uint32_t g = 0;
      for (int u = cta; u < U; u += G) {
        const int4 tl = p.tiles[u / MTU];
        const int mt = PAIR ? 2 * (u % MTU) + rk : u % MTU;
        const uint8_t* wsrc = p.wbank + ((size_t)tl.z * MT + mt) * (size_t)KS * W_BYTES;
        // pair mode: this CTA's half of the tile's rows (N is a multiple of 32)
        const int rows = PAIR ? tl.w >> 1 : tl.w;
        const int row0 = tl.x + (PAIR ? rk * rows : 0);
        const CUtensorMap* map = &maps.m[(rows >> 4) - 1];
        const uint32_t tx = (uint32_t)rows * (BK * 2) + W_BYTES;  // two boxes of `rows` rows x 128 bytes
        for (int s = 0; s < KS; ++s, ++g) {
          if ((int)(g % N_PROD) != pi) continue;
          const uint32_t sl = g % S;
          wait_any<PAIR>(&empty[sl], ((g / S) & 1u) ^ 1u, abort_flag, p.status);
          if (*abort_flag) continue;
          uint8_t* st = base + sl * STAGE_BYTES;
          mbar_expect_tx(&full[sl], tx);
          tma_load_2d(st, map, s * BK, row0, &full[sl]);
          tma_load_2d(st + SUB_BYTES, map, s * BK + 64, row0, &full[sl]);
          bulk_g2s(st + TOK_BYTES, wsrc + (size_t)s * W_BYTES, (uint32_t)W_BYTES, &full[sl]);
          if (g >= gtail) tail_issued |= 1u << (g - gtail);
        }
      }
      // no copy may still be in flight into this CTA's shared memory at exit
      for (uint32_t h = gtail; h < gend; ++h)
        if (tail_issued & (1u << (h - gtail))) mbar_wait_bounded(&full[h % S], (h / S) & 1u, p.status, kWaitLimit);
    }
  } else if ((warp >= W_EPI && warp < W_EPI + 4) || warp >= W_EPI2) {
    // two sets of four epilogue warps (one per TMEM lane quarter each) take
    // alternate passes of 32 token columns, each set with its own staging
    // area and named barrier; every warp releases the accumulator after its
    // set's last TMEM read of the unit (tempty counts 8)
    const int q = warp & 3, set = warp >= W_EPI2 ? 1 : 0;
    const int bid = set ? 3 : 1;
    uint16_t* xch = reinterpret_cast<uint16_t*>(base + XCH_OFF + set * XCH_BYTES);
    const uint16_t* stab = reinterpret_cast<const uint16_t*>(base + STAB_OFF);
    uint32_t* srow = reinterpret_cast<uint32_t*>(base + SROW_OFF);
    const int et = q * 32 + lane;
    int i = 0;
    for (int u = cta; u < U; u += G, ++i) {
      const int4 tl = p.tiles[u / MTU];
      const int mt = PAIR ? 2 * (u % MTU) + rk : u % MTU, cnt = tl.y, N = tl.w;
      const int acc = i & 1;
      // down with an output order: the tile's destination rows are fetched
      // before the accumulator wait (latency off the epilogue's path)
      uint32_t r0 = 0, r1 = 0;
      const bool permuted = MODE == 1 && p.order != nullptr;
      // gate/up: the tile's column scales 2^p (the tokens' pre-scale undone),
      // fetched before the accumulator wait and shared through smem
      float cs0 = 1.0f, cs1 = 1.0f;
      if (MODE == 0 && set == 0) {
        if (et < cnt) cs0 = __int_as_float((127 + __ldg(p.tok_exp + tl.x + et)) << 23);
        if (et + 128 < cnt) cs1 = __int_as_float((127 + __ldg(p.tok_exp + tl.x + et + 128)) << 23);
      }
      if (permuted && set == 0) {
        r0 = et < cnt ? p.order[tl.x + et] : 0u;
        r1 = et + 128 < cnt ? p.order[tl.x + et + 128] : 0u;
        if (p.peer_out) {
          // (owning rank << 28) | row within that rank's buffer
          r0 = ((r0 / p.peer_rows) << 28) | (r0 % p.peer_rows);
          r1 = ((r1 / p.peer_rows) << 28) | (r1 % p.peer_rows);
        }
      }
      wait_any<PAIR>(&tfull[acc], (uint32_t)((i >> 1) & 1), abort_flag, p.status);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t t0 = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * NMAX);
      bool released = false;
      if (permuted) {
        // srow belongs to both sets: set 0 writes it once the previous unit's
        // stores of both sets are done (the 256-thread barrier 4 brackets it)
        named_sync(4, 256);
        if (set == 0) {
          srow[et] = r0;
          if (et + 128 < NMAX) srow[et + 128] = r1;
        }
        named_sync(4, 256);
      }
      float* cscale = reinterpret_cast<float*>(srow);  // gate/up: srow holds the column scales
      if (MODE == 0) {
        named_sync(4, 256);
        if (set == 0) {
          cscale[et] = cs0;
          if (et + 128 < NMAX) cscale[et + 128] = cs1;
        }
        named_sync(4, 256);
      }
      for (int cb = set * XCH_COLS; cb < N; cb += 2 * XCH_COLS) {
        const int nc = min(XCH_COLS, N - cb);
        __syncwarp();
        named_sync(bid, 128);  // this set's xch is free: its previous pass has been consumed
        // round the rows to bf16 (two columns per conversion) into xch[t][row]
        for (int c0 = 0; c0 < nc; c0 += 16) {
          uint32_t v[16];
          tmem_ld16(t0 + cb + c0, v);
          float csc[16];
          if (MODE == 0) {
            // the 16 columns' scales (broadcast 16-byte loads)
            const float4* c4 = reinterpret_cast<const float4*>(cscale + cb + c0);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float4 f = c4[j];
              csc[4 * j] = f.x;
              csc[4 * j + 1] = f.y;
              csc[4 * j + 2] = f.z;
              csc[4 * j + 3] = f.w;
            }
          }
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          if (MODE == 0) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) * csc[j]);
          }
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            const uint32_t pr = pack_bf16x2(__uint_as_float(v[j]), __uint_as_float(v[j + 1]));
            xch[(c0 + j) * MW + et] = (uint16_t)pr;
            xch[(c0 + j + 1) * MW + et] = (uint16_t)(pr >> 16);
          }
        }
        if (cb + 2 * XCH_COLS >= N) {
          // this set's last TMEM read of the accumulator: hand it back
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[acc]);  // local (the odd CTA's are relayed)
          released = true;
        }
        __syncwarp();
        named_sync(bid, 128);  // xch complete
        const int rows = min(nc, cnt - cb);
        if (MODE == 0) {
          // act[t][f] = bf16(silu(g) * u) for g = row f, u = row 64 + f: 8
          // features per chunk, SiLU from the exact window (or chain), one
          // bf16x2 multiply per pair
          uint16_t* act = p.out + (size_t)(tl.x + cb) * p.ldo + mt * 64;
          for (int idx = et; idx < rows * 8; idx += 128) {
            const int t = idx >> 3, f8 = (idx & 7) * 8;
            const uint4 gq = *reinterpret_cast<const uint4*>(xch + t * MW + f8);
            const uint4 uq = *reinterpret_cast<const uint4*>(xch + t * MW + 64 + f8);
            const uint32_t gw[4] = {gq.x, gq.y, gq.z, gq.w}, uw[4] = {uq.x, uq.y, uq.z, uq.w};
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t sp = silu_lookup_bits(stab, gw[j] & 0xffffu) | (silu_lookup_bits(stab, gw[j] >> 16) << 16);
              o[j] = bmul2(sp, uw[j]);
            }
            *reinterpret_cast<uint4*>(act + (size_t)t * p.ldo + f8) = make_uint4(o[0], o[1], o[2], o[3]);
          }
        } else {
          // y row of sorted row tl.x + cb + t: itself, or its (token, slot)
          // position when an output order is given
          if (p.peer_out) {
            // expert parallel: each row goes straight to its source rank's
            // buffer over NVLink (plain 16-byte peer stores)
            for (int idx = et; idx < rows * 16; idx += 128) {
              const int t = idx >> 4, c = (idx & 15) * 8;
              const uint32_t dr = srow[cb + t];
              uint16_t* y = p.peer_out[dr >> 28];
              *reinterpret_cast<uint4*>(y + mt * MW + (size_t)(dr & 0x0fffffffu) * p.ldo + c) =
                  *reinterpret_cast<const uint4*>(xch + t * MW + c);
            }
          } else {
            uint16_t* y = p.out + mt * MW;
            for (int idx = et; idx < rows * 16; idx += 128) {
              const int t = idx >> 4, c = (idx & 15) * 8;
              const size_t row = permuted ? (size_t)srow[cb + t] : (size_t)(tl.x + cb + t);
              *reinterpret_cast<uint4*>(y + row * p.ldo + c) = *reinterpret_cast<const uint4*>(xch + t * MW + c);
            }
          }
        }
      }
      if (!released) {
        // no pass for this set (N <= 32): release at once
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
      }
    }
    // peer stores are visible system-wide before the kernel completes (the
    // expert-parallel barrier that follows on the stream publishes them)
    if (MODE == 1 && p.peer_out) __threadfence_system();
  } else if (warp >= W_DQ) {
    // dequantizers: all eight warps take every stage (a stage's weights are
    // ready half as long after its slot frees up as with alternating
    // groups); warp group grp converts K half grp of the stage: thread =
    // weight row r (TMEM lane), 64 K values -> 32 columns of slot g % SA
    const int grp = (warp - W_DQ) >> 2, q = warp & 3;
    const int r = 32 * q + lane;
    const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16) + kACol + (uint32_t)(grp * 32);
    uint32_t g = 0;
    for (int u = cta; u < U; u += G) {
      for (int s = 0; s < KS; ++s, ++g) {
        const uint32_t sl = g % S, as = g % SA;
        wait_bar(&full[sl], (g / S) & 1u, abort_flag, p.status);
        wait_any<PAIR>(&aempty[as], ((g / SA) & 1u) ^ 1u, abort_flag, p.status);
        const uint8_t* wst = base + sl * STAGE_BYTES + TOK_BYTES;
        const uint32_t sw = *reinterpret_cast<const uint32_t*>(wst + MW * 64 + r * 8 + grp * 4);
        const uint4 c0 = *reinterpret_cast<const uint4*>(wst + (2 * grp) * 2048 + r * 16);
        const uint4 c1 = *reinterpret_cast<const uint4*>(wst + (2 * grp + 1) * 2048 + r * 16);
        uint32_t o[32];
        if (MODE == 0) {
          // f16: E2M1 pair -> f16x2 in hardware, times |scale| in f16 (exact)
          const uint32_t s0 = f16_scale2(sw & 0xffu), s1 = f16_scale2((sw >> 8) & 0xffu);
          const uint32_t s2 = f16_scale2((sw >> 16) & 0xffu), s3 = f16_scale2(sw >> 24);
          dq_word_f16(c0.x, s0, o + 0);
          dq_word_f16(c0.y, s0, o + 4);
          dq_word_f16(c0.z, s1, o + 8);
          dq_word_f16(c0.w, s1, o + 12);
          dq_word_f16(c1.x, s2, o + 16);
          dq_word_f16(c1.y, s2, o + 20);
          dq_word_f16(c1.z, s3, o + 24);
          dq_word_f16(c1.w, s3, o + 28);
        } else {
          const uint32_t s0 = bf16_scale2(sw & 0xffu), s1 = bf16_scale2((sw >> 8) & 0xffu);
          const uint32_t s2 = bf16_scale2((sw >> 16) & 0xffu), s3 = bf16_scale2(sw >> 24);
          dq_word(c0.x, s0, o + 0);
          dq_word(c0.y, s0, o + 4);
          dq_word(c0.z, s1, o + 8);
          dq_word(c0.w, s1, o + 12);
          dq_word(c1.x, s2, o + 16);
          dq_word(c1.y, s2, o + 20);
          dq_word(c1.z, s3, o + 24);
          dq_word(c1.w, s3, o + 28);
        }
        tmem_st32(trow + as * 64, o);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[as]);  // local (the odd CTA's are relayed)
      }
    }
  } else if (PAIR && rk == 1 && (warp == W_MMA || warp == W_MMA2)) {
    // relays of the odd CTA (whose MMA warps are otherwise idle): one
    // cluster-scope arrive per stage (warp W_MMA2: weights in TMEM) or per
    // unit (warp W_MMA: accumulator read) on the even CTA's barrier, once
    // this CTA's eight warps have arrived on its own.  A cluster-scope
    // release arrive costs a warp ~1,000 cycles; paid here, it stays off the
    // dequantizers' and epilogue's per-stage path.
    if (lane == 0) {
      if (warp == W_MMA2) {
        uint32_t g = 0;
        for (int u = cta; u < U; u += G)
          for (int s = 0; s < KS; ++s, ++g) {
            const uint32_t as = g % SA;
            wait_bar(&afull[as], (g / SA) & 1u, abort_flag, p.status);
            if (*abort_flag) break;
            arrive_leader(&afull[as]);
          }
      } else {
        int i = 0;
        for (int u = cta; u < U; u += G, ++i) {
          const int acc = i & 1;
          wait_bar(&tempty[acc], (uint32_t)((i >> 1) & 1), abort_flag, p.status);
          if (*abort_flag) break;
          arrive_leader(&tempty[acc]);
        }
      }
    }
  }

  if (PAIR && rk == 1 && warp == W_MMA && lane == 0) {
    // every MMA of the pair (they write this CTA's TMEM) has completed
    if (!mbar_wait_bounded(&drain, 0, p.status, kWaitLimit)) *abort_flag = 1;
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  // pair mode: neither CTA leaves (or frees its TMEM) while the other may
  // still arrive on its barriers
  if (PAIR) cluster_sync_all();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == W_MMA) {
    if (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------- helpers
// Token tiles: expert e's n_e sorted rows split into ceil(n_e / NMAX) tiles
// of near-equal size (the first n_e % t tiles one row longer), in expert
// order.  One CTA of 1024 threads (E <= 1024).
__global__ void __launch_bounds__(1024) make_tiles_kernel(const uint32_t* __restrict__ offsets, int E,
                                                          int4* __restrict__ tiles, int* __restrict__ ntiles,
                                                          int round) {
  __shared__ int s_warp[32];
  const int e = threadIdx.x, lane = e & 31, w = e >> 5;
  int n = 0, t = 0;
  if (e < E) {
    n = (int)(offsets[e + 1] - offsets[e]);
    t = (n + NMAX - 1) / NMAX;
  }
  // inclusive scan of the tile counts: within each warp, then over the warps
  int inc = t;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += v;
  }
  if (lane == 31) s_warp[w] = inc;
  __syncthreads();
  if (w == 0) {
    int wi = s_warp[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += v;
    }
    s_warp[lane] = wi;
  }
  __syncthreads();
  inc += w > 0 ? s_warp[w - 1] : 0;
  const int start = inc - t;
  if (t > 0) {
    const int b = n / t, rem = n % t;
    for (int i = 0; i < t; ++i) {
      const int cnt = b + (i < rem ? 1 : 0);
      tiles[start + i] = make_int4((int)offsets[e] + i * b + min(i, rem), cnt, e, (cnt + round - 1) & ~(round - 1));
    }
  }
  if (e == 1023) *ntiles = inc;
}

// dst[p] = src[order[p] / k]: 16-bit rows copied into expert order, one warp
// per row (16-byte chunks, four loads in flight per lane).
__global__ void __launch_bounds__(256) gather_rows_kernel(const uint16_t* __restrict__ src,
                                                          const uint32_t* __restrict__ order, int k, int64_t rows,
                                                          int K, uint16_t* __restrict__ dst) {
  const int64_t p = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (p >= rows) return;
  const uint32_t t = order[p] / (uint32_t)k;
  const uint4* s4 = reinterpret_cast<const uint4*>(src + (int64_t)t * K);
  uint4* d4 = reinterpret_cast<uint4*>(dst + p * K);
  const int chunks = K / 8;
  int c = lane;
  for (; c + 96 < chunks; c += 128) {
    const uint4 a = __ldg(s4 + c), b = __ldg(s4 + c + 32), e = __ldg(s4 + c + 64), f = __ldg(s4 + c + 96);
    d4[c] = a;
    d4[c + 32] = b;
    d4[c + 64] = e;
    d4[c + 96] = f;
  }
  for (; c < chunks; c += 32) d4[c] = __ldg(s4 + c);
}

// dst[p] = src[order[p] / k] as scaled f16 (row_to_scaled_f16), one warp per
// row.
template <int CPL>
__global__ void __launch_bounds__(256) gather_rows_f16_kernel(const uint16_t* __restrict__ src,
                                                              const uint32_t* __restrict__ order, int k, int64_t rows,
                                                              int K, uint16_t* __restrict__ dst, int* __restrict__ xexp) {
  const int64_t p = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (p >= rows) return;
  const uint32_t t = order[p] / (uint32_t)k;
  row_to_scaled_f16<CPL>(src + (int64_t)t * K, K, dst + p * K, xexp + p, threadIdx.x & 31);
}

// Prefill bank.  Block (e, m, s) of W_BYTES covers weight rows 128m.. (gate/up:
// rows 0..63 the gate features 64m.., rows 64..127 the same up features;
// down: hidden rows 128m..) over K range 128s..128s+127: codes
// [chunk c][row r][16 bytes] = bytes 16c..16c+15 of the row's 64-byte K
// slice (low nibble first, as in the MLX layout), then [row r][8] scale bytes
// (f16 bits of |scale| >> 7; negative scales flip the sign bits of their
// group's codes).  Gate/up blocks first, then down blocks.
__global__ void prepare_prefill_kernel(const uint8_t* __restrict__ gcodes, const uint8_t* __restrict__ gscales,
                                       const uint8_t* __restrict__ ucodes, const uint8_t* __restrict__ uscales,
                                       const uint8_t* __restrict__ dcodes, const uint8_t* __restrict__ dscales, int E,
                                       int H, int F, uint8_t* __restrict__ bank) {
  const int64_t gu_blocks = (int64_t)E * (F / 64) * (H / BK);  // K stages of BK = 128
  const int64_t blk = blockIdx.x;
  const int r = threadIdx.x;  // MW threads: one weight row each
  int64_t crow;
  const uint8_t *cb, *sbp;
  int K, s;
  if (blk < gu_blocks) {
    const int nst = H / BK, nm = F / 64;
    const int64_t e = blk / ((int64_t)nm * nst);
    const int m = (int)((blk / nst) % nm);
    s = (int)(blk % nst);
    K = H;
    crow = e * F + (int64_t)m * 64 + (r & 63);
    cb = r < 64 ? gcodes : ucodes;
    sbp = r < 64 ? gscales : uscales;
  } else {
    const int64_t b2 = blk - gu_blocks;
    const int nst = F / BK, nm = H / MW;
    const int64_t e = b2 / ((int64_t)nm * nst);
    const int m = (int)((b2 / nst) % nm);
    s = (int)(b2 % nst);
    K = F;
    crow = e * H + (int64_t)m * MW + r;
    cb = dcodes;
    sbp = dscales;
  }
  uint8_t* dst = bank + blk * (int64_t)W_BYTES;
  const uint8_t* code = cb + crow * (K / 2) + (int64_t)s * (BK / 2);
  const uint8_t* scl = sbp + crow * (K / 16) + (int64_t)s * (BK / 16);
  uint32_t sc[2] = {0u, 0u};
#pragma unroll
  for (int gq = 0; gq < 8; ++gq) sc[gq >> 2] |= (uint32_t)prepared_scale_byte(scl[gq]) << (8 * (gq & 3));
#pragma unroll
  for (int wq = 0; wq < 16; ++wq) {
    uint32_t w = *reinterpret_cast<const uint32_t*>(code + 4 * wq);
    if (scl[wq >> 1] & 0x80u) w ^= 0x88888888u;
    reinterpret_cast<uint32_t*>(dst + (wq >> 2) * 2048 + r * 16)[wq & 3] = w;
  }
  reinterpret_cast<uint2*>(dst + MW * 64)[r] = make_uint2(sc[0], sc[1]);
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// Tensor maps of a bf16 [rows][cols] row-major tensor, 128-byte swizzle, box
// 64 x 16(i+1) (one 64-wide K sub-tile of a stage).  Encoded once per (base, rows, cols) and cached: the maps
// only describe the buffer, so a reused workspace hits the cache.
int token_maps(const void* base, uint64_t rows, uint64_t cols, TokMaps* out) {
  struct Entry {
    const void* base;
    uint64_t rows, cols;
    TokMaps maps;
  };
  static std::mutex mu;
  static std::vector<Entry> cache;
  std::lock_guard<std::mutex> lock(mu);
  for (const Entry& en : cache)
    if (en.base == base && en.rows == rows && en.cols == cols) {
      *out = en.maps;
      return B2_OK;
    }
  auto enc = tensor_map_encoder();
  B2_REQUIRE(enc != nullptr, "[prefill grouped gemm] cuTensorMapEncodeTiled is not available from the driver");
  B2_REQUIRE(reinterpret_cast<uintptr_t>(base) % 16 == 0 && (cols * 2) % 16 == 0,
             "[prefill grouped gemm] token rows must be 16-byte aligned");
  Entry en;
  en.base = base;
  en.rows = rows;
  en.cols = cols;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t estr[2] = {1, 1};
  for (int i = 0; i < kMaps; ++i) {
    const cuuint32_t box[2] = {64u, (cuuint32_t)(16 * (i + 1))};  // 128 bytes: the swizzle span
    const CUresult r = enc(&en.maps.m[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                           box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    B2_REQUIRE(r == CUDA_SUCCESS, "[prefill grouped gemm] tensor map encoding failed (%d)", (int)r);
  }
  if (cache.size() >= 16) cache.erase(cache.begin());
  cache.push_back(en);
  *out = en.maps;
  return B2_OK;
}

}  // namespace

size_t prefill_bank_bytes(const b2_moe_block* blk) {
  const size_t E = blk->n_experts, H = blk->hidden, F = blk->ffn;
  return E * ((F / 64) * (H / BK) + (H / MW) * (F / BK)) * (size_t)W_BYTES;
}

bool prefill_gemm_supported(const b2_moe_block* blk) {
  return blk->hidden % 128 == 0 && blk->hidden <= 4096 && blk->ffn % 128 == 0 && blk->n_experts <= 1024;
}

int prepare_prefill(const b2_moe_block* blk, void* dst, cudaStream_t st) {
  (void)silu_table(st);  // setup call: build the SiLU table outside any capture
  const int64_t E = blk->n_experts, H = blk->hidden, F = blk->ffn;
  const int64_t blocks = E * (F / 64) * (H / BK) + E * (H / MW) * (F / BK);
  B2_REQUIRE(blocks <= INT32_MAX, "[prepare_prefill_bank] too many blocks");
  prepare_prefill_kernel<<<(unsigned)blocks, MW, 0, st>>>(
      reinterpret_cast<const uint8_t*>(blk->gate_codes), blk->gate_scales,
      reinterpret_cast<const uint8_t*>(blk->up_codes), blk->up_scales,
      reinterpret_cast<const uint8_t*>(blk->down_codes), blk->down_scales, (int)E, (int)H, (int)F,
      static_cast<uint8_t*>(dst));
  B2_CHECK_LAUNCH("prepare_prefill_bank");
  return B2_OK;
}

int64_t max_tiles(int64_t E, int64_t rows) { return E + rows / NMAX + 1; }

bool pair_mode(const b2_moe_block* blk) {
  // opt-in: measured slower than single-CTA tiles at config 3 (322 vs 299 us
  // per block: each stage's copies took ~7,900 cycles to land in pair mode,
  // ~2,700 in single mode)
  static const bool on = [] {
    const char* v = std::getenv("B2_PREFILL_PAIR");
    return v && v[0] == '1';
  }();
  // both GEMMs of a block share the tiles, so both weight-block counts
  // (gate/up F/64, down H/128) must be even
  return on && (blk->ffn / 64) % 2 == 0 && (blk->hidden / MW) % 2 == 0;
}

int make_tiles(const uint32_t* offsets, int E, int4* tiles, int* ntiles, bool pair, cudaStream_t st) {
  make_tiles_kernel<<<1, 1024, 0, st>>>(offsets, E, tiles, ntiles, pair ? 32 : 16);
  B2_CHECK_LAUNCH("make_tiles");
  return B2_OK;
}

int gather_rows(const uint16_t* src, const uint32_t* order, int k, int64_t rows, int K, uint16_t* dst,
                cudaStream_t st) {
  if (rows == 0 || K == 0) return B2_OK;
  gather_rows_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(src, order, k, rows, K, dst);
  B2_CHECK_LAUNCH("gather_rows");
  return B2_OK;
}

int gather_rows_f16(const uint16_t* src, const uint32_t* order, int k, int64_t rows, int K, uint16_t* dst, int* xexp,
                    cudaStream_t st) {
  if (rows == 0 || K == 0) return B2_OK;
  B2_REQUIRE(K % 8 == 0, "[prefill gather] row length must be a multiple of 8");
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  if (K == 2048)
    gather_rows_f16_kernel<8><<<blocks, 256, 0, st>>>(src, order, k, rows, K, dst, xexp);
  else if (K == 1024)
    gather_rows_f16_kernel<4><<<blocks, 256, 0, st>>>(src, order, k, rows, K, dst, xexp);
  else if (K == 4096)
    gather_rows_f16_kernel<16><<<blocks, 256, 0, st>>>(src, order, k, rows, K, dst, xexp);
  else
    gather_rows_f16_kernel<0><<<blocks, 256, 0, st>>>(src, order, k, rows, K, dst, xexp);
  B2_CHECK_LAUNCH("gather_rows_f16");
  return B2_OK;
}

int expert_gemm(int mode, const b2_moe_block* blk, const uint16_t* tok, int64_t rows, const int4* tiles,
                const int* ntiles, uint16_t* out, const uint32_t* out_order, cudaStream_t st, uint16_t* const* peer_out,
                uint32_t peer_rows, const int* tok_exp) {
  if (rows == 0) return B2_OK;
  B2_REQUIRE(mode == 1 || tok_exp != nullptr, "[prefill grouped gemm] the gate/up GEMM needs the token exponents");
  B2_REQUIRE(peer_out == nullptr || (mode == 1 && out_order != nullptr && peer_rows > 0 && peer_rows < (1u << 28)),
             "[prefill grouped gemm] invalid peer output table");
  Params p;
  const int64_t E = blk->n_experts, H = blk->hidden, F = blk->ffn;
  p.wbank = static_cast<const uint8_t*>(blk->prefill_bank);
  if (mode == 1) p.wbank += (size_t)E * (F / 64) * (H / BK) * W_BYTES;
  p.tiles = tiles;
  p.ntiles = ntiles;
  p.out = out;
  p.silu_tab = mode == 0 ? silu_table(st) : nullptr;
  p.order = mode == 1 ? out_order : nullptr;
  p.peer_out = mode == 1 ? peer_out : nullptr;
  p.peer_rows = peer_rows;
  p.tok_exp = mode == 0 ? tok_exp : nullptr;
  p.status = device_status_ptr();
  B2_REQUIRE(p.status != nullptr, "[prefill grouped gemm] device status word unavailable");
  p.MT = mode == 0 ? (int)(F / 64) : (int)(H / MW);
  p.KS = mode == 0 ? (int)(H / BK) : (int)(F / BK);
  p.ldo = mode == 0 ? (int)F : (int)H;
  TokMaps maps;
  int rc = token_maps(tok, (uint64_t)rows, (uint64_t)(mode == 0 ? H : F), &maps);
  if (rc) return rc;
  const bool pair = pair_mode(blk);
  const void* fn = pair ? (mode == 0 ? (const void*)expert_gemm_kernel<0, true> : (const void*)expert_gemm_kernel<1, true>)
                        : (mode == 0 ? (const void*)expert_gemm_kernel<0, false> : (const void*)expert_gemm_kernel<1, false>);
  const int smem = pair ? Geo<true>::SMEM : Geo<false>::SMEM;
  rc = ensure_dynamic_smem(fn, (size_t)smem, "prefill grouped gemm");
  if (rc) return rc;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  void* args[] = {&p, &maps};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(pair ? sms / 2 * 2 : sms));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = pair ? 1 : 0;
  return check_cuda(cudaLaunchKernelExC(&cfg, fn, args), "prefill grouped gemm");
}

}  // namespace pf
}  // namespace b2
