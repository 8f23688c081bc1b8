// Expert-parallel MoE prefill block over NVLink peer memory.
//
// Rank r of P owns the E/P experts the placement puts on it (contiguous
// ranges [r*E/P, (r+1)*E/P) by default; any permutation the caller passes,
// e.g. one balanced by measured expert load) and a shard of T tokens; the
// router weight is replicated.  The reference runtime has no expert
// parallelism (its MLX collectives have no all-to-all: MLX
// distributed/nccl/nccl.cpp); the block's arithmetic is the single-GPU
// prefill's (RM:9867-10187 sorted branch, SWL:476-524), so every rank's output
// equals b2_moe_block_forward on its own tokens bit for bit.
//
// One forward on every rank, all on the caller's stream, no host round trip:
//   1. stage x into this rank's exported token buffer (peers read it);
//   2. router logits + top-k of the local tokens; the expert ids land in the
//      exported routing buffer;
//   3. barrier A (flags in peer memory, bounded wait): every rank's tokens
//      and routing are in place;
//   4. dispatch: each of the P*T*k (token, slot) rows of all ranks, its id
//      read over NVLink, gets its local expert id if this rank owns the
//      expert, else a discard bin; every peer token with at least one owned
//      row is copied here once (one NVLink read per (token, rank), not per
//      row; the copies run on a side stream while the keys are sorted);
//      stable counting sort over E/P + 1 bins; token tiles;
//   5. gather: the owned rows' tokens, from local memory, in expert order;
//   6. gate/up grouped GEMM + SwiGLU, down grouped GEMM whose epilogue stores
//      each row into the SOURCE rank's exported output buffer at its (token,
//      slot) position (16-byte peer stores);
//   7. barrier B: every rank's expert outputs have landed;
//   8. ordered weighted combine of the local tokens (+ routed scale,
//      + residual) from the local output buffer.
// Two barriers per call are enough for buffer reuse across calls: a rank
// overwrites its token / routing buffers (call i+1, steps 1-2) only after
// barrier B of call i, which every peer reaches after its last read of them
// (step 4 of call i); it writes a peer's output buffer (call i+1, step 6)
// only after barrier A of call i+1, which that peer reaches after its combine
// of call i.
//
// Peer buffers are CUDA IPC mappings of one cudaMalloc region per rank (no
// multicast objects, no TMA from peer memory: the grouped GEMM's TMA loads
// read the local gathered rows only).  Every cross-GPU wait is bounded by
// %globaltimer and records B2_STATUS_WAIT_TIMEOUT instead of hanging.
#include <algorithm>
#include <cstring>
#include <new>
#include <vector>

#include "moe.cuh"
#include "moe_prefill.cuh"
#include "moe_prefill_gemm.cuh"
#include "router.cuh"

namespace b2 {
namespace ep {

constexpr int kMaxRanks = B2_EP_MAX_RANKS;
constexpr uint32_t kHandleMagic = 0xB2E90001u;

// One rank's exported description (B2_EP_HANDLE_BYTES bytes).
struct Handle {
  cudaIpcMemHandle_t ipc;
  uint32_t magic;
  int32_t rank, world, pad;
  int64_t tokens_cap, hidden, n_experts, top_k;
  uint64_t sym_bytes;
};
static_assert(sizeof(Handle) <= B2_EP_HANDLE_BYTES, "handle size");

// Per-rank views of the exported regions (peer pointers for other ranks).
struct Peers {
  const uint16_t* x[kMaxRanks];     // token rows [T][H]
  const uint32_t* inds[kMaxRanks];  // expert ids [T*k]
  uint32_t* flags[kMaxRanks];       // arrival flags [kMaxRanks]
};

// Layout of the exported region (same offsets on every rank).
struct SymLayout {
  size_t flags, inds, x, y, bytes;
};

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

static SymLayout sym_layout(int64_t T, int64_t H, int64_t k) {
  SymLayout l{};
  size_t off = 0;
  l.flags = off;
  off += align256(kMaxRanks * sizeof(uint32_t));
  l.inds = off;
  off += align256((size_t)T * k * 4);
  l.x = off;
  off += align256((size_t)T * H * 2);
  l.y = off;
  off += align256((size_t)T * k * H * 2);
  l.bytes = off;
  return l;
}

// ---------------------------------------------------------------- kernels
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Every rank writes this barrier's epoch into slot `rank` of every rank's
// flag array, then waits until its own array holds the epoch from every rank.
// The epoch is a per-rank device counter advanced once per barrier (all ranks
// run the same barriers, so their counters agree).  Bounded: gives up after
// limit_ns and records B2_STATUS_WAIT_TIMEOUT.
__global__ void __launch_bounds__(32) ep_barrier_kernel(Peers pe, int rank, int world, uint32_t* counter,
                                                        const uint32_t* my_flags, unsigned* status,
                                                        unsigned long long limit_ns) {
  const int lane = threadIdx.x;
  uint32_t e = 0;
  if (lane == 0) {
    e = *counter + 1u;
    *counter = e;
  }
  e = __shfl_sync(0xffffffffu, e, 0);
  // this rank's earlier peer stores (previous kernels fenced them; this one
  // orders the flag after everything the stream did before)
  __threadfence_system();
  if (lane < world) st_release_sys(pe.flags[lane] + rank, e);
  bool ok = true;
  if (lane < world) {
    const uint64_t t0 = globaltimer();
    while ((int32_t)(ld_acquire_sys(my_flags + lane) - e) < 0) {
      if (globaltimer() - t0 > limit_ns) {
        ok = false;
        break;
      }
      __nanosleep(100);
    }
  }
  if (!ok) report_status(status, B2_STATUS_WAIT_TIMEOUT);
  __syncwarp();
  __threadfence_system();
}

// Keys and dispatch in one pass, one warp per token of any rank (token
// tg = q*T + t): lanes 0..k-1 read the token's expert ids from rank q's
// routing buffer and write the keys of its rows (local expert slot under
// the placement, or the discard bin El); if any of them is owned here and the token lives on a
// peer, the warp copies the token row once over NVLink (16-byte L2-coherent
// loads) into x_all[tg] -- one copy per (token, owning rank), however many
// of the token's experts this rank owns.
// KEYS / COPY select the two halves: with more than one rank the keys (then
// the sort) run on the caller's stream while the copies run on a side
// stream -- the sort does not need the rows, only the gather does.
template <bool KEYS, bool COPY>
__global__ void __launch_bounds__(256) ep_dispatch_kernel(Peers pe, int world, int64_t T, int k, int E, int El,
                                                          int rank, int H, const uint32_t* __restrict__ slot_of,
                                                          uint32_t* __restrict__ keys, uint16_t* __restrict__ x_all,
                                                          unsigned* status) {
  const int64_t tg = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (tg >= (int64_t)world * T) return;
  const int q = (int)(tg / T);
  const int64_t t = tg - (int64_t)q * T;
  if (!KEYS && q == rank) return;  // own tokens: nothing to copy
  bool owned = false;
  if (lane < k) {
    const uint32_t e = __ldcv(pe.inds[q] + t * k + lane);
    uint32_t key = (uint32_t)El;
    if (e >= (uint32_t)E) {
      if (KEYS) report_status(status, B2_STATUS_BAD_INDEX);
    } else {
      const uint32_t sl = __ldg(slot_of + e);  // placement: rank-major slot of expert e
      if ((int)(sl / (uint32_t)El) == rank) {
        key = sl % (uint32_t)El;
        owned = true;
      }
    }
    if (KEYS) keys[tg * k + lane] = key;
  }
  if (!COPY || q == rank || !__any_sync(0xffffffffu, owned)) return;
  const uint4* s4 = reinterpret_cast<const uint4*>(pe.x[q] + t * H);
  uint4* d4 = reinterpret_cast<uint4*>(x_all + tg * H);
  const int chunks = H / 8;
  int c = lane;
  for (; c + 96 < chunks; c += 128) {
    const uint4 a = __ldcg(s4 + c), b = __ldcg(s4 + c + 32), d = __ldcg(s4 + c + 64), f = __ldcg(s4 + c + 96);
    d4[c] = a;
    d4[c + 32] = b;
    d4[c + 64] = d;
    d4[c + 96] = f;
  }
  for (; c < chunks; c += 32) d4[c] = __ldcg(s4 + c);
}

// xs[p] = token row of sorted row p for p < offsets[El] (the owned rows) as
// the gate/up GEMM's pre-scaled f16 (pf::row_to_scaled_f16; exponent in
// xexp[p]), read from local memory (pe.x: this rank's tokens and the
// dispatch copies).  One warp per row.
template <int CPL>
__global__ void __launch_bounds__(256) ep_gather_kernel(Peers pe, const uint32_t* __restrict__ order,
                                                        const uint32_t* __restrict__ offsets, int El, int k,
                                                        int64_t T, int H, uint16_t* __restrict__ xs,
                                                        int* __restrict__ xexp) {
  const int64_t p = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (p >= (int64_t)offsets[El]) return;
  const int64_t tg = order[p] / (uint32_t)k;
  const int q = (int)(tg / T);
  const int64_t t = tg - (int64_t)q * T;
  pf::row_to_scaled_f16<CPL>(pe.x[q] + t * H, H, xs + p * H, xexp + p, threadIdx.x & 31);
}

}  // namespace ep
}  // namespace b2

// Opaque context (b2moe.h).
struct b2_ep_ctx {
  int dev = -1, rank = 0, world = 1;
  int64_t T = 0, E = 0, El = 0, H = 0, F = 0, k = 0;
  unsigned long long limit_ns = 0;
  b2_moe_block router{};  // full router (n_experts = E); bank fields unused
  b2_moe_block local{};   // this rank's El experts with their prepared prefill bank
  b2::ep::SymLayout sl{};
  uint8_t* sym = nullptr;                       // exported region
  uint8_t* peer_base[B2_EP_MAX_RANKS] = {};     // per rank (own = sym)
  bool opened[B2_EP_MAX_RANKS] = {};
  bool connected = false;
  // local scratch
  uint8_t* local_mem = nullptr;
  uint8_t* own_bank = nullptr;  // prepared prefill bank when the caller gave none
  float* logits = nullptr;
  float* weights = nullptr;
  uint32_t *keys = nullptr, *order = nullptr, *sorted = nullptr, *inverse = nullptr, *offsets = nullptr,
           *sort_scratch = nullptr, *counter = nullptr;
  int4* tiles = nullptr;
  int* ntiles = nullptr;
  uint16_t *xs = nullptr, *act = nullptr;
  int* xexp = nullptr;  // per gathered row: f16 pre-scale exponent
  uint16_t* x_all = nullptr;  // [world*T][H]: peers' tokens this rank needs (dispatch copies)
  uint32_t* slot_of = nullptr;  // [E]: expert placement (rank-major slot of each expert)
  uint8_t* shared_scratch = nullptr;  // shared expert of the local tokens (if the block has one)
  uint16_t** ytab = nullptr;  // device table: each rank's output buffer
  cudaEvent_t phase[B2_EP_PHASE_EVENTS] = {};
  bool timed = false;
  // side stream of the dispatch copies (more than one rank): forked after
  // barrier A, joined before the gather
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};

namespace b2 {
namespace ep {

static int with_device(const b2_ep_ctx* c) {
  int cur = -1;
  cudaError_t e = cudaGetDevice(&cur);
  if (e != cudaSuccess) return check_cuda(e, "ep");
  if (cur != c->dev) return set_error(B2_ERR_INVALID_ARGUMENT, "[ep] context belongs to device %d, current is %d",
                                      c->dev, cur);
  return B2_OK;
}

static void release(b2_ep_ctx* c) {
  for (int i = 0; i < B2_EP_PHASE_EVENTS; ++i)
    if (c->phase[i]) cudaEventDestroy(c->phase[i]);
  if (c->fork) cudaEventDestroy(c->fork);
  if (c->join) cudaEventDestroy(c->join);
  if (c->side) cudaStreamDestroy(c->side);
  for (int q = 0; q < B2_EP_MAX_RANKS; ++q)
    if (c->opened[q]) cudaIpcCloseMemHandle(c->peer_base[q]);
  if (c->sym) cudaFree(c->sym);
  if (c->local_mem) cudaFree(c->local_mem);
  if (c->own_bank) cudaFree(c->own_bank);
  delete c;
}

static Peers peers(const b2_ep_ctx* c, const uint16_t* x_self) {
  Peers pe{};
  for (int q = 0; q < c->world; ++q) {
    uint8_t* b = c->peer_base[q];
    pe.x[q] = q == c->rank ? x_self : reinterpret_cast<const uint16_t*>(b + c->sl.x);
    pe.inds[q] = reinterpret_cast<const uint32_t*>(b + c->sl.inds);
    pe.flags[q] = reinterpret_cast<uint32_t*>(b + c->sl.flags);
  }
  return pe;
}

static int barrier(const b2_ep_ctx* c, const Peers& pe, cudaStream_t st) {
  if (c->world == 1) return B2_OK;  // no peer to wait for; stream order suffices
  ep_barrier_kernel<<<1, 32, 0, st>>>(pe, c->rank, c->world, c->counter,
                                      reinterpret_cast<const uint32_t*>(c->sym + c->sl.flags), device_status_ptr(),
                                      c->limit_ns);
  B2_CHECK_LAUNCH("ep barrier");
  return B2_OK;
}

static int mark(const b2_ep_ctx* c, int i, cudaStream_t st) {
  if (!c->timed) return B2_OK;
  return check_cuda(cudaEventRecord(c->phase[i], st), "ep phase event");
}

}  // namespace ep
}  // namespace b2

extern "C" {

int b2_ep_create(const b2_moe_block* blk, const b2_ep_config* cfg, b2_ep_ctx** out, void* handle) {
  using namespace b2;
  B2_REQUIRE(out != nullptr && handle != nullptr && cfg != nullptr, "[ep_create] null argument");
  *out = nullptr;
  int rc = validate_block(blk, "ep_create");
  if (rc) return rc;
  const int world = cfg->world, rank = cfg->rank;
  B2_REQUIRE(world >= 1 && world <= B2_EP_MAX_RANKS, "[ep_create] world size must be in [1, %d] (got %d)",
             B2_EP_MAX_RANKS, world);
  B2_REQUIRE(rank >= 0 && rank < world, "[ep_create] rank %d outside [0, %d)", rank, world);
  B2_REQUIRE(blk->n_experts % world == 0, "[ep_create] %lld experts do not divide over %d ranks",
             (long long)blk->n_experts, world);
  B2_REQUIRE(cfg->tokens_per_rank > 0 && cfg->tokens_per_rank * world * blk->top_k <= ((int64_t)1 << 27),
             "[ep_create] tokens_per_rank must be positive and world * tokens * top_k <= 2^27");
  B2_REQUIRE(blk->router_w != nullptr, "[ep_create] router weight is NULL");
  b2_moe_block local = *blk;
  local.n_experts = blk->n_experts / world;
  local.decode_bank = nullptr;
  local.shared_gate_codes = nullptr;  // the shared expert runs on the source rank, not with the routed experts
  B2_REQUIRE(pf::prefill_gemm_supported(&local), "[ep_create] hidden %% 128 and ffn %% 128 must be 0");
  int dev = 0;
  rc = check_cuda(cudaGetDevice(&dev), "ep_create");
  if (rc) return rc;
  b2_ep_ctx* c = new (std::nothrow) b2_ep_ctx();
  if (!c) return set_error(B2_ERR_CUDA, "[ep_create] out of host memory");
  c->dev = dev;
  c->rank = rank;
  c->world = world;
  c->T = cfg->tokens_per_rank;
  c->E = blk->n_experts;
  c->El = local.n_experts;
  c->H = blk->hidden;
  c->F = blk->ffn;
  c->k = blk->top_k;
  c->limit_ns = (unsigned long long)(cfg->wait_timeout_ms > 0 ? cfg->wait_timeout_ms : 10000) * 1000000ull;
  c->router = *blk;
  c->sl = ep::sym_layout(c->T, c->H, c->k);
  auto fail = [&](int code) {
    ep::release(c);
    return code;
  };
  // exported region: zero flags before any peer can see it
  rc = check_cuda(cudaMalloc(&c->sym, c->sl.bytes), "ep_create: cudaMalloc");
  if (rc) return fail(rc);
  rc = check_cuda(cudaMemset(c->sym, 0, c->sl.bytes), "ep_create: cudaMemset");
  if (rc) return fail(rc);
  // local scratch
  const int64_t n = (int64_t)world * c->T * c->k;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += ep::align256(bytes);
    return o;
  };
  const size_t o_logits = take((size_t)c->T * c->E * 4), o_w = take((size_t)c->T * c->k * 4),
               o_keys = take((size_t)n * 4), o_order = take((size_t)n * 4), o_sorted = take((size_t)n * 4),
               o_inv = take((size_t)n * 4), o_offs = take((size_t)(c->El + 2) * 4),
               o_ss = take(gather_sort_scratch_bytes(n, c->El + 1)),
               o_tiles = take((size_t)pf::max_tiles(c->El, n) * sizeof(int4)), o_nt = take(4), o_cnt = take(4),
               o_ytab = take(B2_EP_MAX_RANKS * sizeof(void*)), o_xs = take((size_t)n * c->H * 2),
               o_act = take((size_t)n * c->F * 2), o_sh = take(shared_scratch_bytes(blk, c->T)),
               o_xall = take(world > 1 ? (size_t)world * c->T * c->H * 2 : 0), o_slot = take((size_t)c->E * 4),
               o_xexp = take((size_t)n * 4);
  rc = check_cuda(cudaMalloc(&c->local_mem, off), "ep_create: cudaMalloc");
  if (rc) return fail(rc);
  rc = check_cuda(cudaMemset(c->local_mem, 0, o_xs), "ep_create: cudaMemset");
  if (rc) return fail(rc);
  uint8_t* L = c->local_mem;
  c->logits = reinterpret_cast<float*>(L + o_logits);
  c->weights = reinterpret_cast<float*>(L + o_w);
  c->keys = reinterpret_cast<uint32_t*>(L + o_keys);
  c->order = reinterpret_cast<uint32_t*>(L + o_order);
  c->sorted = reinterpret_cast<uint32_t*>(L + o_sorted);
  c->inverse = reinterpret_cast<uint32_t*>(L + o_inv);
  c->offsets = reinterpret_cast<uint32_t*>(L + o_offs);
  c->sort_scratch = reinterpret_cast<uint32_t*>(L + o_ss);
  c->tiles = reinterpret_cast<int4*>(L + o_tiles);
  c->ntiles = reinterpret_cast<int*>(L + o_nt);
  c->counter = reinterpret_cast<uint32_t*>(L + o_cnt);
  c->ytab = reinterpret_cast<uint16_t**>(L + o_ytab);
  c->xs = reinterpret_cast<uint16_t*>(L + o_xs);
  c->act = reinterpret_cast<uint16_t*>(L + o_act);
  c->shared_scratch = L + o_sh;
  c->x_all = world > 1 ? reinterpret_cast<uint16_t*>(L + o_xall) : nullptr;
  c->slot_of = reinterpret_cast<uint32_t*>(L + o_slot);
  c->xexp = reinterpret_cast<int*>(L + o_xexp);
  {
    std::vector<uint32_t> slots((size_t)c->E);
    std::vector<char> seen((size_t)c->E, 0);
    for (int64_t e = 0; e < c->E; ++e) {
      const int64_t sl = cfg->expert_slot ? cfg->expert_slot[e] : e;
      if (sl < 0 || sl >= c->E || seen[(size_t)sl])
        return fail(set_error(B2_ERR_INVALID_ARGUMENT, "[ep_create] expert_slot is not a permutation of [0, %lld)",
                              (long long)blk->n_experts));
      seen[(size_t)sl] = 1;
      slots[(size_t)e] = (uint32_t)sl;
    }
    rc = check_cuda(cudaMemcpy(c->slot_of, slots.data(), slots.size() * 4, cudaMemcpyHostToDevice),
                    "ep_create: placement");
    if (rc) return fail(rc);
  }
  // the local experts' prepared prefill bank
  if (!local.prefill_bank) {
    const size_t nb = pf::prefill_bank_bytes(&local);
    rc = check_cuda(cudaMalloc(&c->own_bank, nb), "ep_create: cudaMalloc");
    if (rc) return fail(rc);
    rc = pf::prepare_prefill(&local, c->own_bank, 0);
    if (rc) return fail(rc);
    local.prefill_bank = c->own_bank;
  }
  c->local = local;
  rc = check_cuda(cudaDeviceSynchronize(), "ep_create");
  if (rc) return fail(rc);
  for (int i = 0; i < B2_EP_PHASE_EVENTS; ++i) {
    rc = check_cuda(cudaEventCreate(&c->phase[i]), "ep_create: cudaEventCreate");
    if (rc) return fail(rc);
  }
  if (world > 1) {
    rc = check_cuda(cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking), "ep_create: side stream");
    if (!rc) rc = check_cuda(cudaEventCreateWithFlags(&c->fork, cudaEventDisableTiming), "ep_create: event");
    if (!rc) rc = check_cuda(cudaEventCreateWithFlags(&c->join, cudaEventDisableTiming), "ep_create: event");
    if (rc) return fail(rc);
  }
  ep::Handle h{};
  if (world > 1) {
    rc = check_cuda(cudaIpcGetMemHandle(&h.ipc, c->sym), "ep_create: cudaIpcGetMemHandle");
    if (rc) return fail(rc);
  }
  h.magic = ep::kHandleMagic;
  h.rank = rank;
  h.world = world;
  h.tokens_cap = c->T;
  h.hidden = c->H;
  h.n_experts = c->E;
  h.top_k = c->k;
  h.sym_bytes = c->sl.bytes;
  std::memset(handle, 0, B2_EP_HANDLE_BYTES);
  std::memcpy(handle, &h, sizeof(h));
  *out = c;
  return B2_OK;
}

int b2_ep_connect(b2_ep_ctx* c, const void* handles) {
  using namespace b2;
  B2_REQUIRE(c != nullptr && handles != nullptr, "[ep_connect] null argument");
  B2_REQUIRE(!c->connected, "[ep_connect] already connected");
  int rc = ep::with_device(c);
  if (rc) return rc;
  const uint8_t* hb = static_cast<const uint8_t*>(handles);
  for (int q = 0; q < c->world; ++q) {
    ep::Handle h;
    std::memcpy(&h, hb + (size_t)q * B2_EP_HANDLE_BYTES, sizeof(h));
    B2_REQUIRE(h.magic == ep::kHandleMagic && h.rank == q && h.world == c->world,
               "[ep_connect] handle %d is not rank %d's handle of a %d-rank context", q, q, c->world);
    B2_REQUIRE(h.tokens_cap == c->T && h.hidden == c->H && h.n_experts == c->E && h.top_k == c->k &&
                   h.sym_bytes == c->sl.bytes,
               "[ep_connect] rank %d was created with different sizes", q);
    if (q == c->rank) {
      c->peer_base[q] = c->sym;
      continue;
    }
    void* p = nullptr;
    rc = check_cuda(cudaIpcOpenMemHandle(&p, h.ipc, cudaIpcMemLazyEnablePeerAccess), "ep_connect: cudaIpcOpenMemHandle");
    if (rc) return rc;
    c->peer_base[q] = static_cast<uint8_t*>(p);
    c->opened[q] = true;
  }
  uint16_t* ytab[B2_EP_MAX_RANKS] = {};
  for (int q = 0; q < c->world; ++q) ytab[q] = reinterpret_cast<uint16_t*>(c->peer_base[q] + c->sl.y);
  rc = check_cuda(cudaMemcpy(c->ytab, ytab, sizeof(ytab), cudaMemcpyHostToDevice), "ep_connect");
  if (rc) return rc;
  c->connected = true;
  return B2_OK;
}

int b2_ep_set_phase_timing(b2_ep_ctx* c, int enable) {
  B2_REQUIRE(c != nullptr, "[ep_set_phase_timing] null context");
  c->timed = enable != 0;
  return B2_OK;
}

int b2_ep_phase_times(b2_ep_ctx* c, float* ms) {
  using namespace b2;
  B2_REQUIRE(c != nullptr && ms != nullptr, "[ep_phase_times] null argument");
  B2_REQUIRE(c->timed, "[ep_phase_times] phase timing is off (b2_ep_set_phase_timing)");
  for (int i = 0; i + 1 < B2_EP_PHASE_EVENTS; ++i) {
    int rc = check_cuda(cudaEventSynchronize(c->phase[i + 1]), "ep_phase_times");
    if (rc) return rc;
    rc = check_cuda(cudaEventElapsedTime(&ms[i], c->phase[i], c->phase[i + 1]), "ep_phase_times");
    if (rc) return rc;
  }
  return B2_OK;
}

int b2_moe_ep_prefill(b2_ep_ctx* c, const uint16_t* x, int64_t tokens, const float* logits,
                      const uint16_t* residual, uint16_t* out, uint32_t* inds, float* weights, b2_stream_t stream) {
  using namespace b2;
  B2_REQUIRE(c != nullptr, "[moe_ep_prefill] null context");
  B2_REQUIRE(c->connected, "[moe_ep_prefill] context is not connected (b2_ep_connect)");
  B2_REQUIRE(tokens == c->T, "[moe_ep_prefill] every call takes tokens_per_rank = %lld tokens on every rank (got %lld)",
             (long long)c->T, (long long)tokens);
  B2_REQUIRE(x != nullptr && out != nullptr, "[moe_ep_prefill] null x/out");
  B2_REQUIRE(reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                 (!residual || reinterpret_cast<uintptr_t>(residual) % 16 == 0),
             "[moe_ep_prefill] x, residual and out must be 16-byte aligned");
  int rc = ep::with_device(c);
  if (rc) return rc;
  unsigned* status = device_status_ptr();
  if (!status) return set_error(B2_ERR_CUDA, "[moe_ep_prefill] device status word unavailable");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t T = c->T, k = c->k, H = c->H, n = (int64_t)c->world * T * k;
  uint32_t* my_inds = reinterpret_cast<uint32_t*>(c->sym + c->sl.inds);
  uint16_t* my_y = reinterpret_cast<uint16_t*>(c->sym + c->sl.y);
  const ep::Peers pe = ep::peers(c, x);
  if ((rc = ep::mark(c, 0, st))) return rc;
  // 1-2: stage the tokens for the peers, route the local tokens
  if (c->world > 1) {
    rc = check_cuda(cudaMemcpyAsync(c->sym + c->sl.x, x, (size_t)T * H * 2, cudaMemcpyDeviceToDevice, st),
                    "moe_ep_prefill: token staging");
    if (rc) return rc;
  }
  if (!logits) {
    rc = launch_router_logits(x, c->router.router_w, c->router.router_w_dtype, T, c->E, H, c->logits, st);
    if (rc) return rc;
  }
  rc = launch_router_topk(logits ? logits : c->logits, c->router.router_bias, c->router.router_mode, T, c->E, (int)k,
                          c->router.renorm, my_inds, c->weights, st);
  if (rc) return rc;
  if ((rc = ep::mark(c, 1, st))) return rc;
  // 3: every rank's tokens and routing are in place
  if ((rc = ep::barrier(c, pe, st))) return rc;
  if ((rc = ep::mark(c, 2, st))) return rc;
  // 4: keys of every rank's rows, and the peers' tokens this rank needs
  // copied here once each (dispatch)
  {
    const int64_t tokens_all = (int64_t)c->world * T;
    const unsigned gd = (unsigned)((tokens_all * 32 + 255) / 256);
    if (c->world > 1) {
      // the peer copies on the side stream, concurrent with the keys, the
      // sort and the tiles on this one
      rc = check_cuda(cudaEventRecord(c->fork, st), "moe_ep_prefill: fork");
      if (!rc) rc = check_cuda(cudaStreamWaitEvent(c->side, c->fork, 0), "moe_ep_prefill: fork");
      if (rc) return rc;
      ep::ep_dispatch_kernel<false, true><<<gd, 256, 0, c->side>>>(pe, c->world, T, (int)k, (int)c->E, (int)c->El,
                                                                   c->rank, (int)H, c->slot_of, c->keys, c->x_all,
                                                                   status);
      B2_CHECK_LAUNCH("moe_ep_prefill: dispatch copies");
      rc = check_cuda(cudaEventRecord(c->join, c->side), "moe_ep_prefill: join");
      if (rc) return rc;
    }
    ep::ep_dispatch_kernel<true, false><<<gd, 256, 0, st>>>(pe, c->world, T, (int)k, (int)c->E, (int)c->El, c->rank,
                                                            (int)H, c->slot_of, c->keys, c->x_all, status);
    B2_CHECK_LAUNCH("moe_ep_prefill: dispatch keys");
  }
  // owned rows in expert order
  rc = launch_gather_sort_ws(c->keys, n, c->El + 1, c->order, c->sorted, c->inverse, c->offsets, c->sort_scratch, st);
  if (rc) return rc;
  rc = pf::make_tiles(c->offsets, (int)c->El, c->tiles, c->ntiles, pf::pair_mode(&c->local), st);
  if (rc) return rc;
  // 5: their tokens into expert order, from local memory (own tokens from x,
  // the peers' from the dispatch copies)
  if (c->world > 1) {
    rc = check_cuda(cudaStreamWaitEvent(st, c->join, 0), "moe_ep_prefill: join");
    if (rc) return rc;
  }
  {
    ep::Peers lp = pe;
    for (int q = 0; q < c->world; ++q)
      if (q != c->rank) lp.x[q] = c->x_all + (size_t)q * T * H;
    const unsigned gb = (unsigned)((n + 7) / 8);
    if (H == 2048)
      ep::ep_gather_kernel<8><<<gb, 256, 0, st>>>(lp, c->order, c->offsets, (int)c->El, (int)k, T, (int)H, c->xs,
                                                  c->xexp);
    else
      ep::ep_gather_kernel<0><<<gb, 256, 0, st>>>(lp, c->order, c->offsets, (int)c->El, (int)k, T, (int)H, c->xs,
                                                  c->xexp);
    B2_CHECK_LAUNCH("moe_ep_prefill: gather");
  }
  if ((rc = ep::mark(c, 3, st))) return rc;
  // 6: experts; the down GEMM stores every row at its source rank
  rc = pf::expert_gemm(0, &c->local, c->xs, n, c->tiles, c->ntiles, c->act, nullptr, st, nullptr, 0, c->xexp);
  if (rc) return rc;
  if ((rc = ep::mark(c, 4, st))) return rc;
  rc = pf::expert_gemm(1, &c->local, c->act, n, c->tiles, c->ntiles, nullptr, c->order, st, c->ytab,
                       (uint32_t)(T * k));
  if (rc) return rc;
  if ((rc = ep::mark(c, 5, st))) return rc;
  // the shared expert of the local tokens, when the block has one (it needs
  // no peer, so it runs before the wait)
  const uint16_t* shared = nullptr;
  rc = shared_forward(&c->router, x, T, c->shared_scratch, &shared, st);
  if (rc) return rc;
  // 7: every rank's outputs for this rank's tokens have landed
  if ((rc = ep::barrier(c, pe, st))) return rc;
  if ((rc = ep::mark(c, 6, st))) return rc;
  // 8: ordered combine of the local tokens (rows in (token, slot) order)
  rc = launch_combine(my_y, nullptr, c->weights, T, (int)k, H, c->router.routed_scale, shared, residual, out, st);
  if (rc) return rc;
  if (inds) {
    rc = check_cuda(cudaMemcpyAsync(inds, my_inds, (size_t)T * k * 4, cudaMemcpyDeviceToDevice, st),
                    "moe_ep_prefill: routing copy");
    if (rc) return rc;
  }
  if (weights) {
    rc = check_cuda(cudaMemcpyAsync(weights, c->weights, (size_t)T * k * 4, cudaMemcpyDeviceToDevice, st),
                    "moe_ep_prefill: routing copy");
    if (rc) return rc;
  }
  return ep::mark(c, 7, st);
}

int b2_ep_destroy(b2_ep_ctx* c) {
  using namespace b2;
  if (!c) return B2_OK;
  int rc = ep::with_device(c);
  if (rc) return rc;
  cudaDeviceSynchronize();
  ep::release(c);
  return B2_OK;
}

}  // extern "C"
