// bsattn_fwd.cu -- block-sparse causal attention forward for B200 (sm_100a), C ABI.
//
// What it computes (semantics of the reference Triton kernel _fwd_csr,
// sissississi-013/usagi kernels/v4_leaderboard_0740ms.py:31-136):
//   for every head bh = b*H + h and 128-row query block qb with q_start = 128*qb < seq_len:
//     off-diagonal key blocks  kb = col_idx[row_start .. row_end-2]   (v4 :78-86), unmasked
//       except query rows >= seq_len (v4 :93);
//     then the diagonal block kb = qb (v4 :107) with mask key<=query, key<seq_len (v4 :111-113);
//     online softmax in base 2 with scores * (scale*log2 e) in fp32 (v4 :91, :95-99),
//     O += fp16(P) * V with fp32 accumulation (v4 :103), o = O / l, lse = m ln2 + ln l (:126-136).
//   Query blocks starting at or past seq_len write o = 0, lse = -inf (v4 :63-68).
//
// How (B200-native design, not a translation of the Triton program):
//   * Persistent CTAs, one per SM.  Work items (bh, qb) are ordered in groups of heads whose K/V
//     fit in L2 and, within a group, by decreasing qb (longest rows first); CTAs take them from a
//     balanced work list (bsattn_plan) or round robin.  Each CTA streams its items' 128x128 tiles
//     through one continuous pipeline: tile t of the CTA uses S buffer t%2, item i uses Q and O
//     buffers i%2, so the next tile's QK^T and the next item's MMAs overlap the current softmax
//     and the previous item's epilogue.
//   * Warp roles (512 threads, four warpgroups; setmaxnreg re-balances the 128 launch registers):
//       WG0 warp 0        TMA producer: Q per item, K/V tiles named by col_idx into a ring
//       WG0 warp 1        tcgen05 P*V issuer and TMEM owner
//       WG0 warp 2        tcgen05 Q*K^T issuer (warp 3 idle)
//       WG1 (warps 4-7)   softmax for keys 0..63 of every tile   (thread t owns query row t)
//       WG2 (warps 8-11)  softmax for keys 64..127 of every tile (same rows; the two halves of a
//                         row exchange their maxima through shared memory)
//       WG3 (warps 12-15) epilogue: o = O / l into a 16 KB 128B-swizzled staging buffer, one TMA
//                         tensor store per 64-column half, lse, frees the O buffer
//     The producer and MMA warps have the lowest warp ids: the warp schedulers favour them over
//     the softmax warps that share their SMSPs, which keeps MMA issue off the critical path.
//     The producer and the two MMA issuers run on lane 0 of their warps alone (one thread
//     issues each TMA copy and each tcgen05.mma); the other lanes wait at the kernel's end.
//   * Tensor memory, 512 columns x 128 lanes x 32 bit:
//       S[b] = Q K^T (fp32) at columns 128 b, b = 0, 1;  O[b] (fp32) at columns 256 + 128 b.
//       P (fp16, two per column) overwrites S[b]: keys 0..63 at columns +0..31 (written by WG1),
//       keys 64..127 at +64..95 (WG2); P*V reads A straight from tensor memory.
//   * MMA issue is split: one warp issues every S(t) = Q K(t)^T (after PV(t-2) finished with the
//     S buffer), another every PV(t); the producer loads tiles in the order K0, K1, V0, K2, V1, ...
//     that the two warps consume them.
//   * Item descriptors (head, query block, seq_len, tile count, CSR row start) are loaded from
//     global memory once, by the producer, and handed to the softmax warpgroups and the MMA
//     issuers through an 8-slot ring in shared memory: no critical role waits on a dependent chain
//     of global loads (work list, then row_ptr and seq_lens) at an item boundary.
//   * Lazy rescale: the running row max m is raised only when a block's max exceeds it by more
//     than kRescaleLog2 (P stays <= 2^8 in fp16); the final o = O/l and lse are exact.
//   * Every mbarrier wait is bounded (globaltimer); on expiry the CTA raises an abort flag, all
//     roles leave their loops, in-flight TMA/MMA work is drained, TMEM is freed and
//     BSATTN_E_TIMEOUT is left in the workspace error word.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "../../include/bsattn.h"
#include "sm100_ptx.cuh"

namespace bsattn {

constexpr int kBlk = 128;                  // query rows / key rows per tile
constexpr int kHd = 128;                   // head dimension
constexpr int kStages = 4;                 // K/V ring depth
constexpr int kTileBytes = kBlk * kHd * 2; // 32 KB fp16 tile
constexpr int kBoxBytes = kTileBytes / 2;  // one TMA box: 128 rows x 64 columns, 128B swizzle
constexpr int kThreads = 512;              // 4 warpgroups
constexpr int kLoadWarp = 0;
constexpr int kMmaWarp = 1;                // P*V issue, TMEM owner
constexpr int kMmaSWarp = 2;               // Q*K^T issue
constexpr int kSoftmaxWarp0 = 4;           // warps 4-7: keys 0..63, warps 8-11: keys 64..127
constexpr int kEpiWarp0 = 12;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kOCol = 256;            // O[0] column; O[1] at kOCol + 128
constexpr float kRescaleLog2 = 8.0f;
constexpr int kPolyEvery = 4;              // every 4th pair of exponentials runs on the FMA pipe
// Lower bound for the teardown waits on in-flight copies and MMAs, whatever timeout_ns is: they
// finish within microseconds, and the CTA must not exit (or free tensor memory) before they do.
constexpr unsigned long long kDrainNs = 100000000ull;
constexpr int kWsInts = 64;                // workspace: int32[64]
// Active-item ring: the producer publishes each active item's descriptor once; the softmax
// warpgroups, both MMA issuers and the producer's V stream read it from shared memory.
constexpr int kItemRing = 8;
constexpr int kItemReaders = 256 + 3;      // softmax threads, S issuer, PV issuer, V stream
constexpr uint32_t kIdescQK = ptx::idesc_f16_f32(128, 128, /*b_mn_major=*/false);
constexpr uint32_t kIdescQKBf16 = ptx::idesc_f16_f32(128, 128, /*b_mn_major=*/false, true);
constexpr uint32_t kIdescPV = ptx::idesc_f16_f32(128, 128, /*b_mn_major=*/true);
// setmaxnreg budgets.  An increase draws only on the registers the block was launched with
// (512 threads x 128), so per SMSP lane-slot (one warp of each warpgroup) the four budgets must
// sum to at most 4 x kLaunchRegs, or the increase never returns.
constexpr uint32_t kLaunchRegs = 128;      // ptxas allocation for __launch_bounds__(512, 1)
constexpr uint32_t kSoftmaxRegs = 168;
constexpr uint32_t kControlRegs = 88;
constexpr uint32_t kEpilogueRegs = 88;
static_assert(2 * kSoftmaxRegs + kControlRegs + kEpilogueRegs <= 4 * kLaunchRegs,
              "register split exceeds the launch allocation");
static_assert(kLaunchRegs * kThreads <= 65536, "launch register total");

// One work item = one (head, query block).  n_steps = 0: inactive (past seq_len); in the
// active-item ring it marks the end of the CTA's items.
struct Item {
  int bh, qb, seq_len, n_steps, row_start;
};

struct alignas(1024) SharedStorage {
  uint8_t q[2][kTileBytes];
  uint8_t kv[kStages][kTileBytes];
  uint8_t ostage[kTileBytes / 2];   // o staging: 128 rows x 64 columns, 128B-swizzled (TMA store)
  float xmax[2][2][kBlk];     // [tile parity][half][row]: partial row maxima
  float stats[2][3][kBlk];    // [item parity]{m, l_half0, l_half1}[row]
  uint64_t q_full[2];
  uint64_t q_empty[2];
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[2];         // S[b] computed
  uint64_t p_rdy[2][2];       // [b][half]: P half stored in S[b] (and O rescaled if needed)
  uint64_t pv_done[2];        // [b]: PV of a tile whose P sits in S[b] completed
  uint64_t xchg[2][4];        // [tile parity][row quarter]: both halves posted their maxima
  uint64_t o_full[2];         // O[b] holds a finished item
  uint64_t o_free[2];         // epilogue done reading O[b] and its stats
  uint64_t stats_rdy[2];      // softmax published stats[b]
  Item items[kItemRing];      // [active item % kItemRing]
  uint64_t item_full[kItemRing];
  uint64_t item_empty[kItemRing];
  uint64_t drain;
  uint64_t unsignalled;       // never arrived on; waited on only by the test hook
  uint32_t tmem_base;
  int abort_flag;
};

struct FwdParams {
  const int32_t* row_ptr;
  const int32_t* col_idx;
  const int32_t* seq_lens;
  void* o;
  float* lse;
  int* ws;
  long long rp_stride;
  long long ci_stride;
  int max_nnz;
  int BH, H, T, nqb;
  int total_items;
  int group_heads;  // heads per item group (their K/V stay in L2 while the group is processed)
  float scale_log2;
  int out_bf16;
  uint32_t idesc_qk;  // Q K^T instruction descriptor: fp16 or bf16 operands, fp32 accumulator
  unsigned long long timeout_ns;
  int test_unsignalled_wait;  // test hook: the QK^T issuer first waits on a barrier nobody signals
  const int32_t* plan;        // optional work list built by bsattn_plan (null: round robin)
  // Analytic rows (window > 0; row_ptr and col_idx unused): row i lists the first `prefix` blocks
  // not covered by the window, then blocks max(0, i - window + 1) .. i.
  int window, prefix;
};


// Item order: heads are taken in groups of group_heads (sized on the host so a group's K and V fit
// in L2 with room to spare); inside a group, bands of decreasing qb (longest causal rows first),
// and inside a band the group's heads.  Item g -> (bh, qb).
__device__ __forceinline__ Item load_item(const FwdParams& p, int g, bool* csr_bad) {
  Item it;
  const int per_group = p.group_heads * p.nqb;
  const int grp = g / per_group;
  const int r = g - grp * per_group;
  const int gh = min(p.group_heads, p.BH - grp * p.group_heads);
  const int band = r / gh;
  it.bh = grp * p.group_heads + (r - band * gh);
  it.qb = p.nqb - 1 - band;
  int sl = p.T;
  if (p.seq_lens != nullptr) sl = min(__ldg(p.seq_lens + it.bh / p.H), p.T);
  it.seq_len = sl;
  it.n_steps = 0;
  it.row_start = 0;
  if (it.qb * kBlk < sl && p.window > 0) {
    // min(i + 1, prefix + window) blocks: rows up to prefix + window - 1 are all of 0 .. i.
    it.n_steps = min(it.qb + 1, p.prefix + p.window);
  } else if (it.qb * kBlk < sl) {
    const int32_t* rp = p.row_ptr + (long long)it.bh * p.rp_stride + it.qb;
    const int rs = __ldg(rp);
    const int re = __ldg(rp + 1);
    int n_off = max(re - rs - 1, 0);  // v4 :85 range(num_kv - 1)
    if (n_off > 0 && (rs < 0 || (long long)rs + n_off > (long long)p.max_nnz)) {
      if (csr_bad) *csr_bad = true;
      n_off = 0;
    }
    it.row_start = rs;
    it.n_steps = n_off + 1;  // + the diagonal, always computed (v4 :107)
  }
  return it;
}

// Key block of step j < n_steps - 1 (an off-diagonal block) of item it.  CSR rows read
// col_idx (v4 :86); an entry out of range sets *csr_bad and is replaced by the diagonal.  Analytic
// rows have a closed form: with n = n_steps, steps j < n - window are prefix blocks j (the global
// phase of the reference's analytic kernel, v1_baseline.py:264-265), the rest the window blocks
// i - (n - 1 - j) (v1_baseline.py:180-181, :282-283).
__device__ __forceinline__ int offdiag_block(const FwdParams& p, const Item& it, int j,
                                             bool* csr_bad) {
  if (p.window > 0) return j < it.n_steps - p.window ? j : it.qb - (it.n_steps - 1 - j);
  int kb = __ldg(p.col_idx + (long long)it.bh * p.ci_stride + it.row_start + j);
  if (kb < 0 || kb >= p.nqb) {
    if (csr_bad) *csr_bad = true;
    kb = it.qb;
  }
  return kb;
}

// The items of this CTA, in processing order.  Without a work list CTA b takes items b, b + grid,
// b + 2 grid, ...  A work list (bsattn_plan) is {magic, grid, total_items, 0}, then grid + 1
// offsets, then item ids: CTA b takes list[off[b] .. off[b+1]).  Every role walks the same
// sequence; a list that does not match this launch, or an id out of range, ends the CTA's work
// and is reported as BSATTN_E_PLAN (every role reads the same entries, so all stop together).
constexpr int32_t kPlanMagic = 0x4e4c5042;
constexpr int kPlanHeader = 4;

struct ItemCursor {
  int k, end;
};

__device__ __forceinline__ void report_plan_error(const FwdParams& p) {
  atomicCAS(p.ws, 0, BSATTN_E_PLAN);
}

__device__ __forceinline__ void cursor_begin(ItemCursor& c, const FwdParams& p) {
  if (p.plan == nullptr) {
    c.k = static_cast<int>(blockIdx.x);
    c.end = p.total_items;
    return;
  }
  const int32_t* h = p.plan;
  const bool hdr = __ldg(h) == kPlanMagic && __ldg(h + 1) == static_cast<int>(gridDim.x) &&
                   __ldg(h + 2) == p.total_items;
  c.k = hdr ? __ldg(h + kPlanHeader + blockIdx.x) : 0;
  c.end = hdr ? __ldg(h + kPlanHeader + blockIdx.x + 1) : 0;
  if (!hdr || c.k < 0 || c.end < c.k || c.end > p.total_items) {
    c.k = c.end = 0;
    report_plan_error(p);
  }
}

// Next item id of this CTA, or -1 when it has none left.
__device__ __forceinline__ int cursor_next(ItemCursor& c, const FwdParams& p) {
  if (c.k >= c.end) return -1;
  if (p.plan == nullptr) {
    const int g = c.k;
    c.k += static_cast<int>(gridDim.x);
    return g;
  }
  const int g = __ldg(p.plan + kPlanHeader + gridDim.x + 1 + c.k);
  ++c.k;
  if (g < 0 || g >= p.total_items) {
    c.k = c.end;
    report_plan_error(p);
    return -1;
  }
  return g;
}

// Walks this CTA's tiles across its active items: tile t = (item counter ii, step j).
struct TileIter {
  ItemCursor cur;
  int g;      // global item index
  int ii;     // active-item counter (buffer parity = ii & 1)
  int j;      // step within the item
  int t;      // tile counter (S buffer parity = t & 1)
  int kb;     // key block of the step (producer only)
  bool valid;
  Item it;
};

__device__ __forceinline__ bool seek_active(TileIter& x, const FwdParams& p, bool* csr_bad) {
  for (;;) {
    x.g = cursor_next(x.cur, p);
    if (x.g < 0) return false;
    x.it = load_item(p, x.g, csr_bad);
    if (x.it.n_steps > 0) return true;
  }
}

__device__ __forceinline__ void tile_begin(TileIter& x, const FwdParams& p, bool* csr_bad) {
  cursor_begin(x.cur, p);
  x.ii = 0;
  x.j = 0;
  x.t = 0;
  x.valid = seek_active(x, p, csr_bad);
}

__device__ __forceinline__ void tile_next(TileIter& x, const FwdParams& p, bool* csr_bad) {
  ++x.t;
  if (x.j + 1 < x.it.n_steps) {
    ++x.j;
    return;
  }
  x.j = 0;
  ++x.ii;
  x.valid = seek_active(x, p, csr_bad);
}


// Barrier 1 over the epilogue warpgroup only (128 threads).
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// Same barrier with an OR over the warpgroup: every thread gets true when any thread passed true.
__device__ __forceinline__ bool epi_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred a, b;\n\tsetp.ne.u32 a, %1, 0;\n\tbar.red.or.pred b, 1, 128, a;"
      "\n\tselp.u32 %0, 1, 0, b;\n\t}"
               : "=r"(r) : "r"(v ? 1u : 0u) : "memory");
  return r != 0;
}

__device__ __forceinline__ void raise_error(const FwdParams& p, int code) {
  atomicCAS(p.ws, 0, code);
}

// Bounded wait: true when the phase completed; false when this CTA aborted or the wait ran
// past p.timeout_ns (then it raises the abort flag and the timeout error).
__device__ __forceinline__ bool wait_slow(uint32_t bar, uint32_t parity, SharedStorage& sh,
                                          const FwdParams& p) {
  const uint64_t t0 = ptx::globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (*reinterpret_cast<volatile int*>(&sh.abort_flag) != 0) return false;
      if (ptx::globaltimer_ns() - t0 > p.timeout_ns) {
        *reinterpret_cast<volatile int*>(&sh.abort_flag) = 1;
        raise_error(p, BSATTN_E_TIMEOUT);
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, SharedStorage& sh,
                                         const FwdParams& p) {
  if (ptx::mbar_test_wait(bar, parity)) return true;  // completed phases cost ~14 cycles
  return wait_slow(bar, parity, sh, p);
}

// Bounded wait executed by a whole warp; the result is the same on every lane.
__device__ __forceinline__ bool wait_warp(uint32_t bar, uint32_t parity, SharedStorage& sh,
                                          const FwdParams& p) {
  return __all_sync(0xffffffffu, wait_bar(bar, parity, sh, p));
}

// Wait used by the producer and MMA roles, which run on lane 0 alone.
__device__ __forceinline__ bool wait_ctl(uint32_t bar, uint32_t parity, SharedStorage& sh,
                                         const FwdParams& p) {
  return wait_bar(bar, parity, sh, p);
}

// Drain wait used during teardown: ignores the abort flag, still bounded in time.
// Its bound is at least kDrainNs, so a very short pipeline timeout cannot cut the drain short.
__device__ __forceinline__ void wait_drain(uint32_t bar, uint32_t parity, const FwdParams& p) {
  const uint64_t bound = p.timeout_ns > kDrainNs ? p.timeout_ns : kDrainNs;
  const uint64_t t0 = ptx::globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (ptx::mbar_try_wait(bar, parity)) return;
    if ((it & 63u) == 0 && ptx::globaltimer_ns() - t0 > bound) {
      raise_error(p, BSATTN_E_TIMEOUT);
      return;
    }
  }
}

// Active-item ring.  The producer's K stream, which reaches every item first, writes the
// descriptor of each active item once (and an n_steps = 0 end marker after the last); the other
// item walkers read it from shared memory instead of reloading the work list, row_ptr and
// seq_lens at every item boundary.  Slot k % kItemRing; item_full completes once per write,
// item_empty once all kItemReaders have read the slot.  The producer leads every reader by at
// most a few tiles (its K/V ring holds four stages) and every active item has at least one tile,
// so a write never waits for a reader that is kItemRing items behind.
__device__ __forceinline__ bool ring_write(SharedStorage& sh, const FwdParams& p, int k,
                                           const Item& it) {
  const int slot = k & (kItemRing - 1);
  if (k >= kItemRing &&
      !wait_ctl(ptx::smem_u32(&sh.item_empty[slot]),
                static_cast<uint32_t>(k / kItemRing + 1) & 1u, sh, p))
    return false;
  sh.items[slot] = it;
  ptx::mbar_arrive(ptx::smem_u32(&sh.item_full[slot]));
  return true;
}

// One reader thread: active item k (false when this CTA aborted).
__device__ __forceinline__ bool ring_read(SharedStorage& sh, const FwdParams& p, int k, Item& it) {
  const int slot = k & (kItemRing - 1);
  if (!wait_ctl(ptx::smem_u32(&sh.item_full[slot]), static_cast<uint32_t>(k / kItemRing) & 1u, sh,
                p))
    return false;
  it = sh.items[slot];
  ptx::mbar_arrive(ptx::smem_u32(&sh.item_empty[slot]));
  return true;
}

// TileIter walks over the ring (for the readers).
__device__ __forceinline__ void ring_tile_begin(TileIter& x, SharedStorage& sh,
                                                const FwdParams& p) {
  x.ii = 0;
  x.j = 0;
  x.t = 0;
  x.valid = ring_read(sh, p, 0, x.it) && x.it.n_steps > 0;
}

__device__ __forceinline__ void ring_tile_next(TileIter& x, SharedStorage& sh, const FwdParams& p) {
  ++x.t;
  if (x.j + 1 < x.it.n_steps) {
    ++x.j;
    return;
  }
  x.j = 0;
  ++x.ii;
  x.valid = ring_read(sh, p, x.ii, x.it) && x.it.n_steps > 0;
}

// ------------------------------------------------------------------------------------------
// Producer warp.  Load order = MMA consumption order: K(0), K(1), then V(t), K(t+2) for
// t = 0, 1, ...; Q of an item right before its first K.  Lane 0 issues the copies.
// ------------------------------------------------------------------------------------------
__device__ void producer_role(SharedStorage& sh, const CUtensorMap* tq, const CUtensorMap* tk,
                              const CUtensorMap* tv, const FwdParams& p, bool leader) {
  bool csr_bad = false;
  const uint64_t pol_kv = ptx::policy_evict_last();
  const uint64_t pol_q = ptx::policy_evict_first();
  TileIter ks, vs;  // ks runs two tiles ahead of vs
  uint32_t q_issued = 0, q_last_parity = 0;  // bit b: Q buffer b
  int stage = 0;
  uint32_t kv_phase = 0;
  uint32_t kv_issued = 0;       // bit i: stage i received at least one load
  uint32_t kv_last_parity = 0;  // bit i: phase parity of the last load into stage i
  const uint32_t q_smem0 = ptx::smem_u32(sh.q[0]);
  const uint32_t kv_smem0 = ptx::smem_u32(sh.kv[0]);
  const uint32_t kv_full0 = ptx::smem_u32(&sh.kv_full[0]);
  const uint32_t kv_empty0 = ptx::smem_u32(&sh.kv_empty[0]);
  bool ok = true;

  auto load_tile = [&](const CUtensorMap* map, int row) -> bool {
    const uint32_t empty = kv_empty0 + stage * 8;
    const uint32_t full = kv_full0 + stage * 8;
    if (!wait_ctl(empty, kv_phase ^ 1u, sh, p)) return false;
    if (leader) {
      const uint32_t dst = kv_smem0 + stage * kTileBytes;
      ptx::mbar_expect_tx(full, kTileBytes);
      ptx::tma_load_3d(dst, map, full, 0, row, 0, pol_kv);
    }
    kv_issued |= 1u << stage;
    kv_last_parity = (kv_last_parity & ~(1u << stage)) | (kv_phase << stage);
    if (++stage == kStages) stage = 0, kv_phase ^= 1u;
    return true;
  };
  // K of tile x (and Q first when x starts an item); remembers the key block for its V.
  auto load_K = [&](TileIter& x) -> bool {
    const int head_row0 = x.it.bh * p.T;
    if (x.j == 0) {
      const int b = x.ii & 1;
      const uint32_t empty = ptx::smem_u32(&sh.q_empty[b]);
      const uint32_t full = ptx::smem_u32(&sh.q_full[b]);
      const uint32_t ph = (static_cast<uint32_t>(x.ii) >> 1) & 1u;
      if (!wait_ctl(empty, ph ^ 1u, sh, p)) return false;
      if (leader) {
        const uint32_t dst = q_smem0 + b * kTileBytes;
        const int row = head_row0 + x.it.qb * kBlk;
        ptx::mbar_expect_tx(full, kTileBytes);
        ptx::tma_load_3d(dst, tq, full, 0, row, 0, pol_q);
      }
        q_issued |= 1u << b;
      q_last_parity = (q_last_parity & ~(1u << b)) | (ph << b);
    }
    int kb = x.it.qb;  // diagonal
    if (x.j < x.it.n_steps - 1) kb = offdiag_block(p, x.it, x.j, &csr_bad);
    x.kb = kb;
    return load_tile(tk, head_row0 + kb * kBlk);
  };

  // vs trails ks by two tiles; its key block is looked up again (for CSR rows an L1 hit).
  auto key_block = [&](const TileIter& x) -> int {
    return x.j < x.it.n_steps - 1 ? offdiag_block(p, x.it, x.j, nullptr) : x.it.qb;
  };
  // ks publishes each new active item (and the end marker) to the item ring.
  tile_begin(ks, p, &csr_bad);
  int published = 0;
  auto publish = [&]() -> bool {
    if (ks.valid) {
      if (ks.j != 0 || ks.ii < published) return true;
      published = ks.ii + 1;
      return ring_write(sh, p, ks.ii, ks.it);
    }
    if (published > ks.ii) return true;  // end marker already written
    published = ks.ii + 1;
    Item end;
    end.bh = end.qb = end.seq_len = end.row_start = 0;
    end.n_steps = 0;
    return ring_write(sh, p, ks.ii, end);
  };
  ok = publish();
  if (ok) ring_tile_begin(vs, sh, p);
  else vs.valid = false;
  for (int i = 0; i < 2 && ok && ks.valid; ++i) {
    ok = load_K(ks);
    tile_next(ks, p, &csr_bad);
    if (ok) ok = publish();
  }
  while (ok && vs.valid) {
    ok = load_tile(tv, vs.it.bh * p.T + key_block(vs) * kBlk);
    if (!ok) break;
    if (ks.valid) {
      ok = load_K(ks);
      tile_next(ks, p, &csr_bad);
      if (ok) ok = publish();
    }
    ring_tile_next(vs, sh, p);
  }
  if (csr_bad && leader) raise_error(p, BSATTN_E_CSR);
  // No TMA write may still be landing in shared memory when the CTA exits.  On a normal run every
  // copy was consumed and these waits return at once; after an abort (here or in another role)
  // the last copies may still be in flight.
  for (int i = 0; i < kStages; ++i)
    if ((kv_issued >> i) & 1u) wait_drain(kv_full0 + i * 8, (kv_last_parity >> i) & 1u, p);
  for (int b = 0; b < 2; ++b)
    if ((q_issued >> b) & 1u)
      wait_drain(ptx::smem_u32(&sh.q_full[b]), (q_last_parity >> b) & 1u, p);
}

// ------------------------------------------------------------------------------------------
// MMA issue, split over two warps so that one warp's barrier waits overlap the other's MMAs
// (tcgen05.mma issue blocks at the tensor pipe's rate; its queue holds only a couple of MMAs):
//   warp kMmaWarp   (PV)  waits V(t) and both halves of P(t), issues O[ii%2] (+)= P(t) V(t)
//   warp kMmaSWarp  (S)   waits Q, K(t) and "PV(t-2) done", issues S[t%2] = Q K(t)^T
// S(t) overwrites the S buffer that held P(t-2), hence the wait on pv_done before it.  Each role
// runs on lane 0 and commits its own MMAs.  Ring positions follow the producer's load order
// K0, K1, V0, K2, V1, K3, ...: K(t) sits at position t for t < 2 and 2t-1 after; V(t) at 2t+2,
// except for the CTA's last tile, whose V follows V(t-1) directly (no K(t+1) exists) at 2t+1.
// Descriptors are advanced by adding (byte offset >> 4) to the start-address field, which never
// carries out of its 14 bits inside 227 KB of shared memory.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void ring_slot(int pos, int& stage, uint32_t& phase) {
  stage = pos % kStages;
  phase = static_cast<uint32_t>(pos / kStages) & 1u;
}

__device__ void mma_s_role(SharedStorage& sh, const FwdParams& p, uint32_t tmem) {
  const uint64_t q_desc0 = ptx::sdesc_sw128(ptx::smem_u32(sh.q[0]), 16, 1024);
  const uint64_t k_desc0 = ptx::sdesc_sw128(ptx::smem_u32(sh.kv[0]), 16, 1024);
  const uint32_t kv_full0 = ptx::smem_u32(&sh.kv_full[0]);
  const uint32_t kv_empty0 = ptx::smem_u32(&sh.kv_empty[0]);
  // Test hook for the timeout path: a wait that can only end by running out of time.
  if (p.test_unsignalled_wait && !wait_ctl(ptx::smem_u32(&sh.unsignalled), 0, sh, p)) return;
  TileIter x;
  ring_tile_begin(x, sh, p);
  while (x.valid) {
    const int qb = x.ii & 1;
    const int sb = x.t & 1;
    int stage;
    uint32_t phase;
    ring_slot(x.t < 2 ? x.t : 2 * x.t - 1, stage, phase);
    if (x.j == 0 &&
        !wait_ctl(ptx::smem_u32(&sh.q_full[qb]), (static_cast<uint32_t>(x.ii) >> 1) & 1u, sh, p))
      return;
    if (!wait_ctl(kv_full0 + stage * 8, phase, sh, p)) return;
    if (x.t >= 2 &&  // PV(t-2) has read the P stored in S[sb]
        !wait_ctl(ptx::smem_u32(&sh.pv_done[sb]), (static_cast<uint32_t>(x.t - 2) >> 1) & 1u, sh, p))
      return;
    ptx::tc_fence_after();
    const uint64_t qd = q_desc0 + static_cast<uint32_t>((qb * kTileBytes) >> 4);
    const uint64_t kd = k_desc0 + static_cast<uint32_t>((stage * kTileBytes) >> 4);
    const uint32_t d = tmem + sb * 128;
#pragma unroll
    for (int kk = 0; kk < kHd / 16; ++kk) {
      const uint32_t off = ((kk >> 2) * kBoxBytes + (kk & 3) * 32) >> 4;
      ptx::mma_ss(d, qd + off, kd + off, p.idesc_qk, kk > 0 ? 1u : 0u);
    }
    ptx::tc_commit(kv_empty0 + stage * 8);
    ptx::tc_commit(ptx::smem_u32(&sh.s_full[sb]));
    if (x.j == x.it.n_steps - 1) ptx::tc_commit(ptx::smem_u32(&sh.q_empty[qb]));
    ring_tile_next(x, sh, p);
  }
}

__device__ void mma_pv_role(SharedStorage& sh, const FwdParams& p, uint32_t tmem) {
  const uint64_t v_desc0 = ptx::sdesc_sw128(ptx::smem_u32(sh.kv[0]), kBoxBytes, 1024);
  const uint32_t kv_full0 = ptx::smem_u32(&sh.kv_full[0]);
  const uint32_t kv_empty0 = ptx::smem_u32(&sh.kv_empty[0]);
  TileIter x, nx;  // nx = the tile after x (tells whether x is the CTA's last tile)
  ring_tile_begin(x, sh, p);
  nx = x;
  if (nx.valid) ring_tile_next(nx, sh, p);
  while (x.valid) {
    const int ob = x.ii & 1;
    const int sb = x.t & 1;
    const uint32_t tph = (static_cast<uint32_t>(x.t) >> 1) & 1u;
    int stage;
    uint32_t phase;
    ring_slot(nx.valid ? 2 * x.t + 2 : 2 * x.t + 1, stage, phase);
    if (!wait_ctl(kv_full0 + stage * 8, phase, sh, p)) return;
    if (x.j == 0 && x.ii >= 2 &&  // O[ob] read out by the epilogue of item ii-2
        !wait_ctl(ptx::smem_u32(&sh.o_free[ob]), ((static_cast<uint32_t>(x.ii) >> 1) + 1u) & 1u, sh,
                  p))
      return;
    if (!wait_ctl(ptx::smem_u32(&sh.p_rdy[sb][0]), tph, sh, p)) return;
    if (!wait_ctl(ptx::smem_u32(&sh.p_rdy[sb][1]), tph, sh, p)) return;
    ptx::tc_fence_after();
    const uint64_t vd = v_desc0 + static_cast<uint32_t>((stage * kTileBytes) >> 4);
    const uint32_t d = tmem + kOCol + ob * 128;
    const uint32_t a = tmem + sb * 128;
#pragma unroll
    for (int kk = 0; kk < kBlk / 16; ++kk) {
      // V is [key][d] with d contiguous: MN-major B operand.  One K step = 16 keys = two 8-row
      // swizzle atoms (2 KB); the second 64-column half of d sits one TMA box later.  P keys
      // 0..63 sit at columns +0..31 of S[sb], keys 64..127 at +64..95.
      ptx::mma_ts(d, a + (kk >> 2) * 64 + (kk & 3) * 8, vd + static_cast<uint32_t>((kk * 2048) >> 4),
                  kIdescPV, (x.j > 0 || kk > 0) ? 1u : 0u);
    }
    ptx::tc_commit(kv_empty0 + stage * 8);
    ptx::tc_commit(ptx::smem_u32(&sh.pv_done[sb]));
    if (x.j == x.it.n_steps - 1) ptx::tc_commit(ptx::smem_u32(&sh.o_full[ob]));
    x = nx;
    if (nx.valid) ring_tile_next(nx, sh, p);
  }
}

// ------------------------------------------------------------------------------------------
// Softmax warpgroup `half` (0: keys 0..63, 1: keys 64..127 of every tile).  Thread t owns query
// row t and TMEM lane t (warp w may only touch lanes 32*(w%4) .. +31); the warp pair (w, w+4)
// covers the same 32 rows and exchanges partial maxima through shared memory (an mbarrier per
// row quarter and tile parity, so the exchange wait is bounded like every other wait).
// ------------------------------------------------------------------------------------------
__device__ void softmax_role(SharedStorage& sh, const FwdParams& p, int half, uint32_t tmem) {
  const int t = threadIdx.x - kSoftmaxWarp0 * 32 - half * 128;
  const int wq = t >> 5;
  const uint32_t lane_addr = tmem + (static_cast<uint32_t>(wq * 32) << 16);
  const float sl2 = p.scale_log2;
  int tile = 0;
  int ii = 0;

  // Active items from the item ring (the epilogue warpgroup writes the inactive ones).
  for (;; ++ii) {
    const int slot = ii & (kItemRing - 1);
    if (!wait_warp(ptx::smem_u32(&sh.item_full[slot]), static_cast<uint32_t>(ii / kItemRing) & 1u,
                   sh, p))
      return;
    const Item it = sh.items[slot];
    ptx::mbar_arrive(ptx::smem_u32(&sh.item_empty[slot]));
    if (it.n_steps == 0) break;
    const int ob = ii & 1;
    const bool row_valid = it.qb * kBlk + t < it.seq_len;
    float m_run = -1e30f;  // v4 :74
    float l_run = 0.0f;

    for (int j = 0; j < it.n_steps; ++j, ++tile) {
      const int sb = tile & 1;
      const uint32_t s_addr = lane_addr + sb * 128 + half * 64;
      if (!wait_warp(ptx::smem_u32(&sh.s_full[sb]), (static_cast<uint32_t>(tile) >> 1) & 1u, sh, p))
        return;
      ptx::tc_fence_after();
      uint32_t sr[64];
      ptx::tmem_ld32(s_addr + 0, sr + 0);
      ptx::tmem_ld32(s_addr + 32, sr + 32);
      ptx::tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 64; ++c) ptx::reg_fence(sr[c]);
      float s[64];
#pragma unroll
      for (int c = 0; c < 64; ++c) s[c] = __uint_as_float(sr[c]);

      // Key 64*half + c is masked when c >= n_keep: the causal diagonal keeps key <= t (v4 :111;
      // with t valid that also keeps key < seq_len, v4 :112), an invalid row keeps nothing (:93).
      const bool diag = (j == it.n_steps - 1);
      const int n_keep = !row_valid ? 0 : (diag ? min(max(t + 1 - 64 * half, 0), 64) : 64);
      if (n_keep < 64) {
#pragma unroll
        for (int c = 0; c < 64; ++c) s[c] = (c < n_keep) ? s[c] : -INFINITY;
      }
      float a0 = s[0], a1 = s[1], a2 = s[2], a3 = s[3];
#pragma unroll
      for (int c = 4; c < 60; c += 8) {
        a0 = ptx::fmax3(a0, s[c + 0], s[c + 1]);
        a1 = ptx::fmax3(a1, s[c + 2], s[c + 3]);
        a2 = ptx::fmax3(a2, s[c + 4], s[c + 5]);
        a3 = ptx::fmax3(a3, s[c + 6], s[c + 7]);
      }
      a0 = ptx::fmax3(a0, s[60], s[61]);
      a1 = ptx::fmax3(a1, s[62], s[63]);
      const float pmax = ptx::fmax3(a0, a1, fmaxf(a2, a3));
      // Row max over both halves (raw scores; scale > 0 commutes with max).
      sh.xmax[tile & 1][half][t] = pmax;
      ptx::mbar_arrive(ptx::smem_u32(&sh.xchg[tile & 1][wq]));
      if (!wait_warp(ptx::smem_u32(&sh.xchg[tile & 1][wq]), (static_cast<uint32_t>(tile) >> 1) & 1u,
                     sh, p))
        return;
      const float m_cand = fmaxf(pmax, sh.xmax[tile & 1][half ^ 1][t]) * sl2;

      // Both halves see the same maxima, so they take the same rescale decision.
      float alpha = 1.0f;
      bool rescale = false;
      if (j == 0) {
        m_run = fmaxf(m_run, m_cand);
      } else {
        const bool need = m_cand > m_run + kRescaleLog2;
        rescale = __any_sync(0xffffffffu, need);
        if (rescale) {
          const float m_new = fmaxf(m_run, m_cand);
          alpha = ptx::ex2(m_run - m_new);
          l_run *= alpha;
          m_run = m_new;
        }
      }
      const uint64_t sc2 = ptx::pack2(sl2, sl2);
      const uint64_t nm2 = ptx::pack2(-m_run, -m_run);
      uint64_t acc0 = 0, acc1 = 0;
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const uint64_t x2 = ptx::ffma2(ptx::pack2(s[2 * i], s[2 * i + 1]), sc2, nm2);
        float x0, x1, p0, p1;
        ptx::unpack2(x2, x0, x1);
        if (kPolyEvery > 0 && (i % kPolyEvery) == kPolyEvery - 1) {
          ptx::exp2_poly_pair(x0, x1, p0, p1);
        } else {
          p0 = ptx::ex2(x0);
          p1 = ptx::ex2(x1);
        }
        const uint64_t p2 = ptx::pack2(p0, p1);
        if (i & 1) acc1 = ptx::fadd2(acc1, p2); else acc0 = ptx::fadd2(acc0, p2);
        __half2 hv = __floats2half2_rn(p0, p1);
        pk[i] = *reinterpret_cast<uint32_t*>(&hv);
      }
      ptx::tmem_st32(s_addr, pk);
      if (rescale) {
        // O must include PV(tile-1) before it is scaled.  pv_done[b] completes once per tile that
        // uses S[b]; PV(tile-3) (same buffer) completed before S(tile-1) was issued, and PV(tile+1)
        // cannot run before this tile's P exists, so the parity below is unambiguous.
        const uint32_t pb = static_cast<uint32_t>(tile - 1) & 1u;
        if (!wait_warp(ptx::smem_u32(&sh.pv_done[pb]), (static_cast<uint32_t>(tile - 1) >> 1) & 1u,
                       sh, p))
          return;
        ptx::tc_fence_after();
        const uint32_t o_addr = lane_addr + kOCol + ob * 128 + half * 64;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t orow[32];
          ptx::tmem_ld32(o_addr + c * 32, orow);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            ptx::reg_fence(orow[i]);
            orow[i] = __float_as_uint(__uint_as_float(orow[i]) * alpha);
          }
          ptx::tmem_st32(o_addr + c * 32, orow);
        }
      }
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      ptx::mbar_arrive(ptx::smem_u32(&sh.p_rdy[sb][half]));
      float l0, l1;
      ptx::unpack2(ptx::fadd2(acc0, acc1), l0, l1);
      l_run += l0 + l1;
    }

    // Publish the row statistics of item ii for the epilogue.  stats[ob] was last read by the
    // epilogue of item ii-2, which released O[ob] through o_free[ob].
    if (ii >= 2) {
      if (!wait_warp(ptx::smem_u32(&sh.o_free[ob]), ((static_cast<uint32_t>(ii) >> 1) + 1u) & 1u,
                     sh, p))
        return;
    }
    if (half == 0) sh.stats[ob][0][t] = m_run;
    sh.stats[ob][1 + half][t] = l_run;
    ptx::mbar_arrive(ptx::smem_u32(&sh.stats_rdy[ob]));
  }
}

// ------------------------------------------------------------------------------------------
// Epilogue warpgroup: o = O / l (v4 :126-133), lse = m ln2 + ln l (v4 :134-136); rows of
// query blocks past seq_len are written as o = 0, lse = -inf (v4 :63-68).
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void store_row32(const FwdParams& p, size_t row, int col0,
                                            const float* v32, float mul, bool valid) {
  uint4 pk[4];
  uint32_t* w = reinterpret_cast<uint32_t*>(pk);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float a = valid ? v32[2 * i] * mul : 0.0f;
    const float b = valid ? v32[2 * i + 1] * mul : 0.0f;
    if (p.out_bf16) {
      __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    } else {
      __half2 h = __floats2half2_rn(a, b);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.o) + row * kHd + col0);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = pk[i];
}

__device__ void epilogue_role(SharedStorage& sh, const FwdParams& p, uint32_t tmem,
                              const CUtensorMap* to) {
  const int t = threadIdx.x - kEpiWarp0 * 32;
  const int wq = t >> 5;
  const uint32_t lane_addr = tmem + (static_cast<uint32_t>(wq * 32) << 16);
  int ii = 0;
  ItemCursor cur;
  cursor_begin(cur, p);
  for (int g = cursor_next(cur, p); g >= 0; g = cursor_next(cur, p)) {
    const Item it = load_item(p, g, nullptr);
    const int q_pos = it.qb * kBlk + t;
    const size_t row = static_cast<size_t>(it.bh) * p.T + q_pos;
    if (it.n_steps == 0) {
      float z[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) z[i] = 0.0f;
#pragma unroll
      for (int c = 0; c < 4; ++c) store_row32(p, row, c * 32, z, 0.0f, false);
      if (p.lse) p.lse[row] = -INFINITY;
      continue;
    }
    const int ob = ii & 1;
    const uint32_t ph = (static_cast<uint32_t>(ii) >> 1) & 1u;
    // The four warps take one decision: the named barriers below need all of them.
    bool ok = wait_warp(ptx::smem_u32(&sh.o_full[ob]), ph, sh, p);
    if (ok) ok = wait_warp(ptx::smem_u32(&sh.stats_rdy[ob]), ph, sh, p);
    if (epi_any(!ok)) return;
    ptx::tc_fence_after();
    const bool row_valid = q_pos < it.seq_len;
    const float m_run = sh.stats[ob][0][t];
    const float l_run = sh.stats[ob][1][t] + sh.stats[ob][2][t];
    const float inv_l = l_run > 0.0f ? 1.0f / l_run : 1.0f;
    const uint32_t o_addr = lane_addr + kOCol + ob * 128;
    const uint32_t stage = ptx::smem_u32(sh.ostage) + static_cast<uint32_t>(t) * 128u;
    const int row0 = it.bh * p.T + it.qb * kBlk;
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {
      if (t == 0) ptx::bulk_wait_read0();  // the previous store has read the staging buffer
      epi_sync();
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t orow[32];
        ptx::tmem_ld32(o_addr + h * 64 + c * 32, orow);
        ptx::tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          ptx::reg_fence(orow[2 * i]);
          ptx::reg_fence(orow[2 * i + 1]);
          const float a = row_valid ? __uint_as_float(orow[2 * i]) * inv_l : 0.0f;
          const float b = row_valid ? __uint_as_float(orow[2 * i + 1]) * inv_l : 0.0f;
          if (p.out_bf16) {
            __nv_bfloat162 v2 = __floats2bfloat162_rn(a, b);
            w[i] = *reinterpret_cast<uint32_t*>(&v2);
          } else {
            __half2 v2 = __floats2half2_rn(a, b);
            w[i] = *reinterpret_cast<uint32_t*>(&v2);
          }
        }
        // 16-byte chunk k of this row lands at chunk k ^ (row % 8): the 128-byte swizzle.
#pragma unroll
        for (int kq = 0; kq < 4; ++kq) {
          const uint32_t chunk = static_cast<uint32_t>((c * 4 + kq) ^ (t & 7));
          ptx::sts128(stage + chunk * 16u, w[4 * kq], w[4 * kq + 1], w[4 * kq + 2], w[4 * kq + 3]);
        }
      }
      ptx::fence_async_smem();
      epi_sync();
      if (t == 0) {
        ptx::tma_store_3d(to, ptx::smem_u32(sh.ostage), 0, row0, h);
        ptx::bulk_commit();
      }
    }
    if (p.lse) {
      p.lse[row] = (row_valid && l_run > 0.0f) ? m_run * 0.69314718055994531f + logf(l_run)
                                               : -INFINITY;
    }
    ptx::tc_fence_before();
    ptx::mbar_arrive(ptx::smem_u32(&sh.o_free[ob]));
    ++ii;
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    bsattn_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                      const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap to,
                      const __grid_constant__ FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = ptx::smem_u32(smem_raw);
  SharedStorage& sh =
      *reinterpret_cast<SharedStorage*>(smem_raw + (((raw + 1023u) & ~1023u) - raw));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(ptx::smem_u32(&sh.q_full[b]), 1);
      ptx::mbar_init(ptx::smem_u32(&sh.q_empty[b]), 1);
      ptx::mbar_init(ptx::smem_u32(&sh.s_full[b]), 1);
      ptx::mbar_init(ptx::smem_u32(&sh.p_rdy[b][0]), 128);
      ptx::mbar_init(ptx::smem_u32(&sh.p_rdy[b][1]), 128);
      ptx::mbar_init(ptx::smem_u32(&sh.o_full[b]), 1);
      ptx::mbar_init(ptx::smem_u32(&sh.o_free[b]), 128);
      ptx::mbar_init(ptx::smem_u32(&sh.stats_rdy[b]), 256);
    }
    for (int i = 0; i < kStages; ++i) {
      ptx::mbar_init(ptx::smem_u32(&sh.kv_full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&sh.kv_empty[i]), 1);
    }
    ptx::mbar_init(ptx::smem_u32(&sh.pv_done[0]), 1);
    ptx::mbar_init(ptx::smem_u32(&sh.pv_done[1]), 1);
    for (int b = 0; b < 2; ++b)
      for (int q = 0; q < 4; ++q) ptx::mbar_init(ptx::smem_u32(&sh.xchg[b][q]), 64);
    for (int i = 0; i < kItemRing; ++i) {
      ptx::mbar_init(ptx::smem_u32(&sh.item_full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&sh.item_empty[i]), kItemReaders);
    }
    ptx::mbar_init(ptx::smem_u32(&sh.drain), 2);  // one commit per MMA-issuing thread
    ptx::mbar_init(ptx::smem_u32(&sh.unsignalled), 1);
    sh.abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kLoadWarp && lane == 0) {
    ptx::tma_prefetch_desc(&tq);
    ptx::tma_prefetch_desc(&tk);
    ptx::tma_prefetch_desc(&tv);
    ptx::tma_prefetch_desc(&to);
  }
  if (warp == kMmaWarp) {
    ptx::tmem_alloc(ptx::smem_u32(&sh.tmem_base), kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = sh.tmem_base;

  if (warp >= kSoftmaxWarp0 && warp < kEpiWarp0) {
    ptx::setmaxnreg_inc<kSoftmaxRegs>();
    softmax_role(sh, p, (warp - kSoftmaxWarp0) >> 2, tmem);
  } else if (warp < kSoftmaxWarp0) {
    ptx::setmaxnreg_dec<kControlRegs>();
    if (warp == kLoadWarp) {
      if (lane == 0) producer_role(sh, &tq, &tk, &tv, p, true);
    } else if (warp == kMmaWarp) {
      if (lane == 0) mma_pv_role(sh, p, tmem);
    } else if (warp == kMmaSWarp) {
      if (lane == 0) mma_s_role(sh, p, tmem);
    }
  } else {
    ptx::setmaxnreg_dec<kEpilogueRegs>();
    epilogue_role(sh, p, tmem, &to);
    if (threadIdx.x == kEpiWarp0 * 32) ptx::bulk_wait0();  // every tile store has completed
  }
  __syncwarp();
  // A role that aborted may have left a tensor-memory load or store of its own in flight.
  ptx::tmem_wait_ld();
  ptx::tmem_wait_st();
  ptx::tc_fence_before();
  __syncthreads();
  // Each MMA-issuing thread commits once more; when both commits have arrived, every MMA of the
  // CTA has completed and the tensor memory can be released.
  if ((warp == kMmaWarp || warp == kMmaSWarp) && lane == 0)
    ptx::tc_commit(ptx::smem_u32(&sh.drain));
  if (warp == kMmaWarp) {
    if (lane == 0) wait_drain(ptx::smem_u32(&sh.drain), 0, p);
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// A [rows, 128] fp16 row-major matrix seen as 3-D {64 columns, rows, 2 column halves} with
// strides {256 B per row, 128 B per half}: one box {64, 128, 2} moves a whole 128x128 tile and
// lands it as two 16 KB blocks (columns 0..63 of all rows, then 64..127), each in the 128-byte
// swizzled K-major layout the MMA descriptors address.
static int make_tile_map(CUtensorMap* map, const void* base, uint64_t rows, bool bf16,
                         uint32_t box_z = 2) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return BSATTN_E_TMA;
  cuuint64_t dims[3] = {64, static_cast<cuuint64_t>(rows), 2};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(kHd * 2), 128};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(kBlk), box_z};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                   const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? BSATTN_OK : BSATTN_E_TMA;
}

struct DeviceInfo {
  int sms = 0;
  int major = 0;
  bool configured = false;
};

static std::mutex g_mu;
static DeviceInfo g_dev[64];
static unsigned long long g_timeout_ns = 2000000000ull;
static int g_test_unsignalled_wait = 0;

static size_t smem_bytes() { return sizeof(SharedStorage) + 1024; }

// Heads per item group: K and V of one head take 2 * T * 128 * 2 bytes; keep a group's worth near
// 32 MB of L2.
static int group_heads_for(int B, int H, int T) {
  const long long head_kv_bytes = 512ll * T;
  return static_cast<int>(
      std::max<long long>(1, std::min<long long>(static_cast<long long>(B) * H,
                                                 (32ll << 20) / head_kv_bytes)));
}

// Host copy of the kernel's item order (load_item): item g -> (bh, qb).
static void item_coords(int g, int BH, int nqb, int group_heads, int* bh, int* qb) {
  const int per_group = group_heads * nqb;
  const int grp = g / per_group;
  const int r = g - grp * per_group;
  const int gh = std::min(group_heads, BH - grp * group_heads);
  const int band = r / gh;
  *bh = grp * group_heads + (r - band * gh);
  *qb = nqb - 1 - band;
}

static int device_setup(int* sms_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return BSATTN_E_CUDA;
  if (dev < 0 || dev >= 64) return BSATTN_E_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceInfo& di = g_dev[dev];
  if (!di.configured) {
    int major = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
      return BSATTN_E_CUDA;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return BSATTN_E_CUDA;
    if (major != 10) return BSATTN_E_DEVICE;
    // The warpgroup register split only works if the kernel was built with the register count
    // it assumes; a smaller launch allocation would make setmaxnreg.inc wait forever.
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, bsattn_fwd_kernel) != cudaSuccess) return BSATTN_E_CUDA;
    if (fa.numRegs != static_cast<int>(kLaunchRegs)) return BSATTN_E_CUDA;
    if (cudaFuncSetAttribute(bsattn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem_bytes())) != cudaSuccess)
      return BSATTN_E_CUDA;
    di.major = major;
    di.sms = sms;
    di.configured = true;
  }
  if (sms_out) *sms_out = di.sms;
  return BSATTN_OK;
}

}  // namespace bsattn

using namespace bsattn;

// ------------------------------------------------------------------------------------------
// bf16 -> fp16 conversion of V.  With bf16 inputs the reference computes Q K^T on bf16 operands
// and P V as fp16(P) . fp16(V) (v4 :103, :123); the tensor cores take both operands of one MMA in
// the same type, so V is converted once, up front, to the fp16 the reference converts it to.
// Eight elements per thread and step (16-byte loads and stores), grid-stride.
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) bf16_to_f16_kernel(const uint4* __restrict__ src,
                                                          uint4* __restrict__ dst, long long n8) {
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n8; i += 256ll * gridDim.x) {
    const uint4 a = src[i];
    const uint32_t in[4] = {a.x, a.y, a.z, a.w};
    uint32_t out[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&in[w]));
      __half2 h = __floats2half2_rn(f.x, f.y);
      out[w] = *reinterpret_cast<uint32_t*>(&h);
    }
    dst[i] = make_uint4(out[0], out[1], out[2], out[3]);
  }
}

extern "C" {

size_t bsattn_workspace_bytes(void) { return kWsInts * sizeof(int); }

int bsattn_version(void) { return 102; }

void bsattn_set_timeout_ns(uint64_t ns) { g_timeout_ns = ns > 0 ? ns : 1; }

int bsattn_bf16_to_f16(const void* src, void* dst, int64_t n, void* stream) {
  if (!src || !dst) return BSATTN_E_NULL;
  if (n < 0 || (n % 8) != 0) return BSATTN_E_SHAPE;
  if ((reinterpret_cast<uintptr_t>(src) & 15u) != 0 || (reinterpret_cast<uintptr_t>(dst) & 15u) != 0)
    return BSATTN_E_ALIGN;
  if (n == 0) return BSATTN_OK;
  int sms = 0;
  const int rc = device_setup(&sms);
  if (rc != BSATTN_OK) return rc;
  const long long n8 = n / 8;
  const int grid = static_cast<int>(std::min<long long>((n8 + 255) / 256, 8ll * sms));
  bf16_to_f16_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), static_cast<uint4*>(dst), n8);
  return cudaGetLastError() == cudaSuccess ? BSATTN_OK : BSATTN_E_CUDA;
}

void bsattn_test_unsignalled_wait(int enable) { g_test_unsignalled_wait = enable ? 1 : 0; }

int bsattn_setup(void) { return device_setup(nullptr); }

const char* bsattn_strerror(int code) {
  switch (code) {
    case BSATTN_OK: return "ok";
    case BSATTN_E_SHAPE: return "bad shape: need B,H >= 1, T % 128 == 0, D == 128";
    case BSATTN_E_ALIGN: return "q/k/v/o must be 16-byte aligned";
    case BSATTN_E_NULL: return "required pointer is NULL";
    case BSATTN_E_WORKSPACE: return "workspace missing or too small";
    case BSATTN_E_CUDA: return "CUDA runtime error";
    case BSATTN_E_TMA: return "TMA descriptor encoding failed";
    case BSATTN_E_DEVICE: return "device is not an sm_100 (B200-class) GPU";
    case BSATTN_E_CSR: return "CSR row_ptr/col_idx entry out of range";
    case BSATTN_E_TIMEOUT: return "kernel pipeline wait timed out";
    case BSATTN_E_DTYPE: return "unsupported dtype flags";
    case BSATTN_E_PLAN: return "work list does not match this call";
    default: return "unknown error";
  }
}

}  // extern "C"

namespace bsattn {

// The row pattern of one call: CSR arrays, or analytic prefix + window rows (window > 0).
struct Pattern {
  const int32_t* row_ptr;
  const int32_t* col_idx;
  int64_t rp_stride, ci_stride;
  int max_nnz;
  int window, prefix;
};

// Checks and launch shared by the CSR and the analytic entry points.
static int launch_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                      const Pattern& pat, const int32_t* seq_lens, int B, int H, int T, int D,
                      float scale, int dtype_flags, const int32_t* plan, int plan_grid,
                      void* workspace, size_t workspace_bytes, void* stream) {
  if (!q || !k || !v || !o) return BSATTN_E_NULL;
  if (B < 1 || H < 1 || T < kBlk || (T % kBlk) != 0 || D != kHd) return BSATTN_E_SHAPE;
  const long long rows = static_cast<long long>(B) * H * T;
  const long long items = static_cast<long long>(B) * H * (T / kBlk);
  if (rows >= (1ll << 31) || items >= (1ll << 30)) return BSATTN_E_SHAPE;
  if ((dtype_flags & ~(BSATTN_OUT_BF16 | BSATTN_IN_BF16)) != 0) return BSATTN_E_DTYPE;
  const bool qk_bf16 = (dtype_flags & BSATTN_IN_BF16) != 0;
  auto misaligned = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) != 0; };
  if (misaligned(q) || misaligned(k) || misaligned(v) || misaligned(o)) return BSATTN_E_ALIGN;
  if (!workspace || workspace_bytes < bsattn_workspace_bytes()) return BSATTN_E_WORKSPACE;
  if (plan != nullptr && ((reinterpret_cast<uintptr_t>(plan) & 3u) != 0 || plan_grid < 1 ||
                          plan_grid > items))
    return BSATTN_E_PLAN;

  int sms = 0;
  int rc = device_setup(&sms);
  if (rc != BSATTN_OK) return rc;

  CUtensorMap tq, tk, tv, to;
  if ((rc = make_tile_map(&tq, q, rows, qk_bf16)) != BSATTN_OK) return rc;
  if ((rc = make_tile_map(&tk, k, rows, qk_bf16)) != BSATTN_OK) return rc;
  if ((rc = make_tile_map(&tv, v, rows, false)) != BSATTN_OK) return rc;
  if ((rc = make_tile_map(&to, o, rows, (dtype_flags & BSATTN_OUT_BF16) != 0, 1)) != BSATTN_OK)
    return rc;

  FwdParams p;
  memset(&p, 0, sizeof(p));
  p.row_ptr = pat.row_ptr;
  p.col_idx = pat.col_idx;
  p.seq_lens = seq_lens;
  p.o = o;
  p.lse = lse;
  p.ws = static_cast<int*>(workspace);
  p.rp_stride = pat.rp_stride;
  p.ci_stride = pat.ci_stride;
  p.max_nnz = pat.max_nnz;
  p.window = pat.window;
  p.prefix = pat.prefix;
  p.BH = B * H;
  p.H = H;
  p.T = T;
  p.nqb = T / kBlk;
  p.total_items = static_cast<int>(items);
  p.group_heads = group_heads_for(B, H, T);
  const double sc = scale > 0.0f ? static_cast<double>(scale) : 1.0 / sqrt(static_cast<double>(D));
  p.scale_log2 = static_cast<float>(sc * 1.4426950408889634);
  p.out_bf16 = (dtype_flags & BSATTN_OUT_BF16) != 0 ? 1 : 0;
  p.idesc_qk = qk_bf16 ? kIdescQKBf16 : kIdescQK;
  p.timeout_ns = g_timeout_ns;
  p.test_unsignalled_wait = g_test_unsignalled_wait;
  p.plan = plan;

  const int grid = plan != nullptr ? plan_grid : static_cast<int>(std::min<long long>(sms, items));
  bsattn_fwd_kernel<<<grid, kThreads, smem_bytes(), static_cast<cudaStream_t>(stream)>>>(tq, tk,
                                                                                        tv, to, p);
  return cudaGetLastError() == cudaSuccess ? BSATTN_OK : BSATTN_E_CUDA;
}

// Largest window / prefix the analytic rows accept (their sum stays far from int overflow).
constexpr int kMaxWindow = 1 << 24;

static int check_window(int window, int global_blocks) {
  if (window < 1 || window > kMaxWindow || global_blocks < 0 || global_blocks > kMaxWindow)
    return BSATTN_E_SHAPE;
  return BSATTN_OK;
}

}  // namespace bsattn

extern "C" {

int bsattn_fwd_plan(const void* q, const void* k, const void* v, void* o, float* lse,
                    const int32_t* row_ptr, const int32_t* col_idx, const int32_t* seq_lens,
                    int B, int H, int T, int D, int64_t rp_stride_bh, int64_t ci_stride_bh,
                    int max_nnz, float scale, int dtype_flags, const int32_t* plan, int plan_grid,
                    void* workspace, size_t workspace_bytes, void* stream) {
  if (!row_ptr || !col_idx) return BSATTN_E_NULL;
  if (max_nnz < 0 || rp_stride_bh < 0 || ci_stride_bh < 0) return BSATTN_E_SHAPE;
  const Pattern pat{row_ptr, col_idx, rp_stride_bh, ci_stride_bh, max_nnz, 0, 0};
  return launch_fwd(q, k, v, o, lse, pat, seq_lens, B, H, T, D, scale, dtype_flags, plan,
                    plan_grid, workspace, workspace_bytes, stream);
}

int bsattn_fwd_window(const void* q, const void* k, const void* v, void* o, float* lse,
                      const int32_t* seq_lens, int B, int H, int T, int D, int window,
                      int global_blocks, float scale, int dtype_flags, const int32_t* plan,
                      int plan_grid, void* workspace, size_t workspace_bytes, void* stream) {
  const int rc = check_window(window, global_blocks);
  if (rc != BSATTN_OK) return rc;
  const Pattern pat{nullptr, nullptr, 0, 0, 0, window, global_blocks};
  return launch_fwd(q, k, v, o, lse, pat, seq_lens, B, H, T, D, scale, dtype_flags, plan,
                    plan_grid, workspace, workspace_bytes, stream);
}

int bsattn_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
               const int32_t* row_ptr, const int32_t* col_idx, const int32_t* seq_lens, int B,
               int H, int T, int D, int64_t rp_stride_bh, int64_t ci_stride_bh, int max_nnz,
               float scale, int dtype_flags, void* workspace, size_t workspace_bytes,
               void* stream) {
  return bsattn_fwd_plan(q, k, v, o, lse, row_ptr, col_idx, seq_lens, B, H, T, D, rp_stride_bh,
                         ci_stride_bh, max_nnz, scale, dtype_flags, nullptr, 0, workspace,
                         workspace_bytes, stream);
}

int bsattn_plan_bytes(int B, int H, int T, int grid, size_t* bytes) {
  if (!bytes) return BSATTN_E_NULL;
  if (B < 1 || H < 1 || T < kBlk || (T % kBlk) != 0) return BSATTN_E_SHAPE;
  const long long items = static_cast<long long>(B) * H * (T / kBlk);
  if (items >= (1ll << 30) || grid < 1 || grid > items) return BSATTN_E_SHAPE;
  *bytes = static_cast<size_t>(kPlanHeader + grid + 1 + items) * sizeof(int32_t);
  return BSATTN_OK;
}

}  // extern "C"

namespace bsattn {

// Work list: items sorted by their tile count, largest first (ties keep the kernel's item order,
// so the big items stay grouped by head for L2 reuse), dealt to the CTAs in a snake order
// (0 .. grid-1, then grid-1 .. 0, ...).  Each CTA keeps its items in that sorted order.
// row_tiles(bh, qb) is the tile count of a live item (query block below seq_len).
template <class RowTiles>
static int build_plan(const int32_t* seq_lens, int B, int H, int T, int grid, int32_t* plan,
                      size_t plan_bytes, RowTiles row_tiles) {
  if (!plan) return BSATTN_E_NULL;
  size_t need = 0;
  int rc = bsattn_plan_bytes(B, H, T, grid, &need);
  if (rc != BSATTN_OK) return rc;
  if (plan_bytes < need) return BSATTN_E_WORKSPACE;
  const int nqb = T / kBlk, BH = B * H;
  const int items = BH * nqb;
  const int gh = group_heads_for(B, H, T);
  std::vector<int> size(items);
  int max_size = 0;
  for (int g = 0; g < items; ++g) {
    int bh, qb;
    item_coords(g, BH, nqb, gh, &bh, &qb);
    int sl = T;
    if (seq_lens) sl = std::min(seq_lens[bh / H], T);
    const int n = qb * kBlk < sl ? row_tiles(bh, qb) : 0;
    size[g] = n;
    max_size = std::max(max_size, n);
  }
  // Counting sort by size, descending and stable.
  std::vector<int> start(max_size + 2, 0);
  for (int g = 0; g < items; ++g) ++start[max_size - size[g] + 1];
  for (int i = 1; i <= max_size + 1; ++i) start[i] += start[i - 1];
  std::vector<int> order(items);
  for (int g = 0; g < items; ++g) order[start[max_size - size[g]]++] = g;
  // Snake deal; CTA c's items keep their sorted order.
  std::vector<int> cta(items), count(grid, 0);
  for (int kpos = 0; kpos < items; ++kpos) {
    const int r = kpos / grid, i = kpos - r * grid;
    cta[kpos] = (r & 1) ? grid - 1 - i : i;
    ++count[cta[kpos]];
  }
  plan[0] = kPlanMagic;
  plan[1] = grid;
  plan[2] = items;
  plan[3] = 0;
  int32_t* off = plan + kPlanHeader;
  int32_t* list = off + grid + 1;
  off[0] = 0;
  for (int c = 0; c < grid; ++c) off[c + 1] = off[c] + count[c];
  std::vector<int> fill(off, off + grid);
  for (int kpos = 0; kpos < items; ++kpos) list[fill[cta[kpos]]++] = order[kpos];
  return BSATTN_OK;
}

}  // namespace bsattn

extern "C" {

// The tile count of a CSR item is the kernel's: the listed off-diagonal blocks plus the diagonal
// (rows whose range does not fit col_idx count as the diagonal alone, as in load_item).
int bsattn_plan(const int32_t* row_ptr, int64_t rp_stride_bh, const int32_t* seq_lens, int B,
                int H, int T, int max_nnz, int grid, int32_t* plan, size_t plan_bytes) {
  if (!row_ptr) return BSATTN_E_NULL;
  if (rp_stride_bh < 0 || max_nnz < 0) return BSATTN_E_SHAPE;
  return build_plan(seq_lens, B, H, T, grid, plan, plan_bytes, [&](int bh, int qb) {
    const int32_t* rp = row_ptr + static_cast<long long>(bh) * rp_stride_bh + qb;
    int n_off = std::max(rp[1] - rp[0] - 1, 0);
    if (n_off > 0 && (rp[0] < 0 || static_cast<long long>(rp[0]) + n_off > max_nnz)) n_off = 0;
    return n_off + 1;
  });
}

// Analytic rows hold min(qb + 1, global_blocks + window) tiles.
int bsattn_plan_window(const int32_t* seq_lens, int B, int H, int T, int window, int global_blocks,
                       int grid, int32_t* plan, size_t plan_bytes) {
  const int rc = check_window(window, global_blocks);
  if (rc != BSATTN_OK) return rc;
  const int L = window + global_blocks;
  return build_plan(seq_lens, B, H, T, grid, plan, plan_bytes,
                    [&](int, int qb) { return std::min(qb + 1, L); });
}

int bsattn_check_error(void* workspace, void* stream, int* status) {
  if (!workspace || !status) return BSATTN_E_NULL;
  int h = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(&h, workspace, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return BSATTN_E_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return BSATTN_E_CUDA;
  if (h != 0) {
    if (cudaMemsetAsync(workspace, 0, sizeof(int), s) != cudaSuccess) return BSATTN_E_CUDA;
    if (cudaStreamSynchronize(s) != cudaSuccess) return BSATTN_E_CUDA;
  }
  *status = h;
  return BSATTN_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------
// Allocation-free entry point.
//
// Some callers cannot allocate device memory at the point they run attention: code executing
// inside a memory pool or arena they do not own, allocators that are locked or exhausted while
// a step is in flight, or C callers with no allocator of their own for CUDA memory.  They cannot
// provide the workspace bsattn_fwd expects, so this entry point supplies it from a fixed array
// of device memory compiled into the library.  It calls no cudaMalloc, cudaFree or other
// allocating routine.
// ------------------------------------------------------------------------------------------
namespace bsattn {

// Scratch for bsattn_fwd_noalloc: 256 bytes, the whole workspace the kernel uses (its error word
// plus reserved space).  It does not grow with B, H or T.  Every GPU that loads this library
// holds one copy until the process exits, and every call on that GPU shares it.
constexpr size_t kNoAllocScratchBytes = 256;
static __device__ __align__(256) int g_noalloc_scratch[kNoAllocScratchBytes / sizeof(int)];

// Device address of g_noalloc_scratch per device; host code must not use the symbol itself.
static void* g_noalloc_addr[64];

static int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return BSATTN_E_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr)
      return BSATTN_E_CUDA;
    g_noalloc_addr[dev] = ptr;
  }
  *out = g_noalloc_addr[dev];
  return BSATTN_OK;
}

}  // namespace bsattn

extern "C" {

int bsattn_fwd_noalloc(const void* q, const void* k, const void* v, void* o, float* lse,
                       const int32_t* row_ptr, const int32_t* col_idx, const int32_t* seq_lens,
                       int B, int H, int T, int D, int64_t rp_stride_bh, int64_t ci_stride_bh,
                       int max_nnz, float scale, int dtype_flags, int* status, void* stream) {
  // The workspace the kernel needs must fit the fixed scratch array.
  if (bsattn_workspace_bytes() > kNoAllocScratchBytes) return BSATTN_E_WORKSPACE;
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc != BSATTN_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The scratch keeps the previous call's contents; the error word must start at zero.
  if (cudaMemsetAsync(scratch, 0, sizeof(int), s) != cudaSuccess) return BSATTN_E_CUDA;
  rc = bsattn_fwd(q, k, v, o, lse, row_ptr, col_idx, seq_lens, B, H, T, D, rp_stride_bh,
                  ci_stride_bh, max_nnz, scale, dtype_flags, scratch, kNoAllocScratchBytes, stream);
  if (rc != BSATTN_OK) return rc;
  if (status != nullptr &&
      cudaMemcpyAsync(status, scratch, sizeof(int), cudaMemcpyDefault, s) != cudaSuccess)
    return BSATTN_E_CUDA;
  return BSATTN_OK;
}

}  // extern "C"
