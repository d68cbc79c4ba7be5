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
//   * Persistent CTAs, one per SM, each running two independent query-tile "slots".  Items
//     (bh, qb) are dealt round-robin in order of decreasing qb, so the longest causal rows go
//     first and every CTA sees the same mix.
//   * Warp roles (384 threads).  setmaxnreg gives the softmax warpgroups 208 registers and the
//     control warpgroup 88; every device function is inlined, because a called function has
//     one register allocation and cannot serve both budgets.
//       warps 0-3  softmax + epilogue for slot 0   (thread t owns query row t of the tile)
//       warps 4-7  softmax + epilogue for slot 1
//       warp  8    TMA producer: Q tiles per item, K/V tiles named by col_idx into a ring
//       warp  9    tcgen05 MMA issuer and TMEM owner
//     The producer and MMA warps run their schedules with all 32 lanes so that addresses and
//     descriptors are warp-uniform (the form TMA and tcgen05.mma take their operands in); only
//     lane 0 issues the copies, MMAs and commits.
//       warps 10-11 idle (they complete warpgroup 2 for the register re-allocation)
//   * Tensor memory (512 columns x 128 lanes x 32 bit):
//       slot s: S = Q K^T (fp32) at columns [256 s, 256 s + 128), O (fp32) at [256 s + 128, 256 s + 256)
//       P (fp16, two per column) overwrites the first 64 columns of S and is the A operand of the
//       P*V MMA straight from tensor memory.
//   * Shared memory: Q[2] (32 KB each) + a ring of kStages K/V tiles (32 KB each), all in the
//     128-byte-swizzled layout TMA writes and the MMA descriptors read.
//   * MMA issue order per slot: S(0); then repeatedly PV(j), S(j+1).  Slots interleave, so while
//     slot 0's softmax runs on S, the tensor core computes slot 1's MMAs, and vice versa.  A
//     commit after S(j+1) therefore also certifies PV(j) done, which lets the softmax warps
//     rescale O in place without another barrier.
//   * Lazy rescale: the running row max m is only raised when a block's max exceeds it by more
//     than kRescaleLog2 (P then stays <= 2^8 in fp16); the final o = O/l and lse are exact.
//   * Every mbarrier wait is bounded (globaltimer); on expiry the CTA raises an abort flag, all
//     roles leave their loops, in-flight TMA/MMA work is drained, TMEM is freed and
//     BSATTN_E_TIMEOUT is left in the workspace error word.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <mutex>

#include "../../include/bsattn.h"
#include "sm100_ptx.cuh"

namespace bsattn {

constexpr int kBlk = 128;                  // query rows / key rows per tile
constexpr int kHd = 128;                   // head dimension
constexpr int kStages = 4;                 // K/V ring depth
constexpr int kTileBytes = kBlk * kHd * 2; // 32 KB fp16 tile
constexpr int kBoxBytes = kTileBytes / 2;  // one TMA box: 128 rows x 64 columns, 128B swizzle
constexpr int kThreads = 384;            // 3 warpgroups
constexpr int kLoadWarp = 8;
constexpr int kMmaWarp = 9;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.0f;
constexpr int kPolyEvery = 4;              // every 4th pair of exponentials runs on the FMA pipe
// setmaxnreg budgets.  The increase draws only on the registers the block was launched with
// (384 threads x 168 = 64512), so per SMSP lane-slot (two softmax warps + one control warp)
// 2 * kSoftmaxRegs + kControlRegs must not exceed 3 * kLaunchRegs, or the increase never returns.
constexpr uint32_t kLaunchRegs = 168;      // ptxas allocation for __launch_bounds__(384, 1)
constexpr uint32_t kSoftmaxRegs = 208;
constexpr uint32_t kControlRegs = 88;
static_assert(2 * kSoftmaxRegs + kControlRegs <= 3 * kLaunchRegs, "register split exceeds launch");
static_assert(kLaunchRegs * kThreads <= 65536, "launch register total");
constexpr int kWsInts = 64;                // workspace: int32[64]
constexpr uint32_t kIdescQK = ptx::idesc_f16_f32(128, 128, /*b_mn_major=*/false);
constexpr uint32_t kIdescPV = ptx::idesc_f16_f32(128, 128, /*b_mn_major=*/true);

struct alignas(1024) SharedStorage {
  uint8_t q[2][kTileBytes];
  uint8_t kv[kStages][kTileBytes];
  uint64_t q_full[2];
  uint64_t q_empty[2];
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[2];
  uint64_t p_lo[2];   // P columns for keys 0..63 stored (and O rescaled if needed)
  uint64_t p_hi[2];   // P columns for keys 64..127 stored
  uint64_t o_full[2];
  uint64_t drain;
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
  float scale_log2;
  int out_bf16;
  unsigned long long timeout_ns;
};

// One work item = one (head, query block).
struct Item {
  int bh, qb, seq_len, n_steps, row_start;
};

// Items are numbered band-major with bands in decreasing qb: item g -> qb = nqb-1 - g/BH.
__device__ __forceinline__ Item load_item(const FwdParams& p, int g, bool* csr_bad) {
  Item it;
  const int band = g / p.BH;
  it.bh = g - band * p.BH;
  it.qb = p.nqb - 1 - band;
  int sl = p.T;
  if (p.seq_lens != nullptr) sl = min(__ldg(p.seq_lens + it.bh / p.H), p.T);
  it.seq_len = sl;
  it.n_steps = 0;
  it.row_start = 0;
  if (it.qb * kBlk < sl) {
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

struct Stream {
  int g;
  int stride;
  int j;
  int kb;
  Item it;
};

__device__ __forceinline__ bool next_active(Stream& s, const FwdParams& p, bool* csr_bad) {
  for (;;) {
    s.g += s.stride;
    if (s.g >= p.total_items) return false;
    s.it = load_item(p, s.g, csr_bad);
    if (s.it.n_steps > 0) {
      s.j = 0;
      return true;
    }
  }
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
  if (ptx::mbar_try_wait(bar, parity)) return true;
  return wait_slow(bar, parity, sh, p);
}

// Drain wait used during teardown: ignores the abort flag, still bounded in time.
__device__ __forceinline__ void wait_drain(uint32_t bar, uint32_t parity, const FwdParams& p) {
  const uint64_t t0 = ptx::globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (ptx::mbar_try_wait(bar, parity)) return;
    if ((it & 63u) == 0 && ptx::globaltimer_ns() - t0 > p.timeout_ns) {
      raise_error(p, BSATTN_E_TIMEOUT);
      return;
    }
  }
}

// Bounded wait executed by a whole warp; the result is the same on every lane.
__device__ __forceinline__ bool wait_warp(uint32_t bar, uint32_t parity, SharedStorage& sh,
                                          const FwdParams& p) {
  return __all_sync(0xffffffffu, wait_bar(bar, parity, sh, p));
}

// ------------------------------------------------------------------------------------------
// Producer warp: mirrors the MMA issue order exactly -- S(first) of slot 0 and 1, then per slot
// "V(j), K(j+1)" -- so the ring holds tiles in the order the MMAs consume them.  The whole warp
// runs the control flow (so coordinates stay warp-uniform, which is what the TMA instruction
// consumes); lane 0 alone issues the copies.
// ------------------------------------------------------------------------------------------
__device__ void producer_role(SharedStorage& sh, const CUtensorMap* tq, const CUtensorMap* tk,
                              const CUtensorMap* tv, const FwdParams& p, bool leader) {
  bool csr_bad = false;
  const uint64_t pol_kv = ptx::policy_evict_last();
  const uint64_t pol_q = ptx::policy_evict_first();
  Stream st[2];
  bool has[2];
  uint32_t qe_phase[2] = {0, 0};
  uint32_t q_issued = 0, q_last_parity = 0;    // bit s: slot s
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
    if (!wait_warp(empty, kv_phase ^ 1u, sh, p)) return false;
    if (leader) {
      const uint32_t dst = kv_smem0 + stage * kTileBytes;
      ptx::mbar_expect_tx(full, kTileBytes);
      ptx::tma_load_2d(dst, map, full, 0, row, pol_kv);
      ptx::tma_load_2d(dst + kBoxBytes, map, full, 64, row, pol_kv);
    }
    __syncwarp();
    kv_issued |= 1u << stage;
    kv_last_parity = (kv_last_parity & ~(1u << stage)) | (kv_phase << stage);
    if (++stage == kStages) stage = 0, kv_phase ^= 1u;
    return true;
  };
  auto load_S = [&](int s) -> bool {
    Stream& x = st[s];
    const int head_row0 = x.it.bh * p.T;
    if (x.j == 0) {
      const uint32_t empty = ptx::smem_u32(&sh.q_empty[s]);
      const uint32_t full = ptx::smem_u32(&sh.q_full[s]);
      if (!wait_warp(empty, qe_phase[s] ^ 1u, sh, p)) return false;
      if (leader) {
        const uint32_t dst = q_smem0 + s * kTileBytes;
        const int row = head_row0 + x.it.qb * kBlk;
        ptx::mbar_expect_tx(full, kTileBytes);
        ptx::tma_load_2d(dst, tq, full, 0, row, pol_q);
        ptx::tma_load_2d(dst + kBoxBytes, tq, full, 64, row, pol_q);
      }
      __syncwarp();
      q_issued |= 1u << s;
      q_last_parity = (q_last_parity & ~(1u << s)) | (qe_phase[s] << s);
      qe_phase[s] ^= 1u;
    }
    int kb = x.it.qb;  // diagonal
    if (x.j < x.it.n_steps - 1) {
      kb = __ldg(p.col_idx + (long long)x.it.bh * p.ci_stride + x.it.row_start + x.j);
      if (kb < 0 || kb >= p.nqb) {
        csr_bad = true;
        kb = x.it.qb;
      }
    }
    x.kb = kb;
    return load_tile(tk, head_row0 + kb * kBlk);
  };
  auto load_V = [&](int s) -> bool { return load_tile(tv, st[s].it.bh * p.T + st[s].kb * kBlk); };

#pragma unroll
  for (int s = 0; s < 2; ++s) {
    st[s].g = 2 * blockIdx.x + s - 2 * gridDim.x;
    st[s].stride = 2 * gridDim.x;
    has[s] = next_active(st[s], p, &csr_bad);
    if (has[s] && ok) ok = load_S(s);
  }
  while (ok && (has[0] || has[1])) {
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      if (!ok || !has[s]) continue;
      ok = load_V(s);
      if (!ok) continue;
      if (st[s].j + 1 < st[s].it.n_steps) {
        ++st[s].j;
        ok = load_S(s);
      } else {
        has[s] = next_active(st[s], p, &csr_bad);
        if (has[s]) ok = load_S(s);
      }
    }
  }
  if (csr_bad && leader) raise_error(p, BSATTN_E_CSR);
  if (!ok) {
    // Aborted: make sure no TMA write is still landing in shared memory before the CTA exits.
    for (int i = 0; i < kStages; ++i)
      if ((kv_issued >> i) & 1u) wait_drain(kv_full0 + i * 8, (kv_last_parity >> i) & 1u, p);
    for (int s = 0; s < 2; ++s)
      if ((q_issued >> s) & 1u)
        wait_drain(ptx::smem_u32(&sh.q_full[s]), (q_last_parity >> s) & 1u, p);
  }
}

// ------------------------------------------------------------------------------------------
// MMA warp: the whole warp runs the schedule and builds the descriptors (warp-uniform values);
// lane 0 issues every tcgen05.mma and tcgen05.commit, so one thread owns all MMA completions.
// Descriptors are formed once and advanced by adding (byte offset >> 4) to the start-address
// field, which never carries out of its 14 bits inside the 227 KB of shared memory.
// ------------------------------------------------------------------------------------------
__device__ void mma_role(SharedStorage& sh, const FwdParams& p, uint32_t tmem, bool leader) {
  Stream st[2];
  bool has[2];
  uint32_t qf_phase[2] = {0, 0};
  uint32_t pr_phase[2] = {0, 0};
  int stage = 0;
  uint32_t kv_phase = 0;
  const uint64_t q_desc0 = ptx::sdesc_sw128(ptx::smem_u32(sh.q[0]), 16, 1024);
  const uint64_t k_desc0 = ptx::sdesc_sw128(ptx::smem_u32(sh.kv[0]), 16, 1024);
  const uint64_t v_desc0 = ptx::sdesc_sw128(ptx::smem_u32(sh.kv[0]), kBoxBytes, 1024);
  const uint32_t kv_full0 = ptx::smem_u32(&sh.kv_full[0]);
  const uint32_t kv_empty0 = ptx::smem_u32(&sh.kv_empty[0]);
  bool ok = true;

  auto issue_S = [&](int s) -> bool {
    Stream& x = st[s];
    if (x.j == 0) {
      if (!wait_warp(ptx::smem_u32(&sh.q_full[s]), qf_phase[s], sh, p)) return false;
      qf_phase[s] ^= 1u;
    }
    if (!wait_warp(kv_full0 + stage * 8, kv_phase, sh, p)) return false;
    ptx::tc_fence_after();
    const uint64_t qd = q_desc0 + static_cast<uint32_t>((s * kTileBytes) >> 4);
    const uint64_t kd = k_desc0 + static_cast<uint32_t>((stage * kTileBytes) >> 4);
    const uint32_t d = tmem + s * 256;
    if (leader) {
#pragma unroll
      for (int kk = 0; kk < kHd / 16; ++kk) {
        const uint32_t off = ((kk >> 2) * kBoxBytes + (kk & 3) * 32) >> 4;
        ptx::mma_ss(d, qd + off, kd + off, kIdescQK, kk > 0 ? 1u : 0u);
      }
      ptx::tc_commit(kv_empty0 + stage * 8);
      ptx::tc_commit(ptx::smem_u32(&sh.s_full[s]));
      if (x.j == x.it.n_steps - 1) ptx::tc_commit(ptx::smem_u32(&sh.q_empty[s]));
    }
    __syncwarp();
    if (++stage == kStages) stage = 0, kv_phase ^= 1u;
    return true;
  };
  auto issue_PV = [&](int s) -> bool {
    Stream& x = st[s];
    if (!wait_warp(kv_full0 + stage * 8, kv_phase, sh, p)) return false;
    const uint64_t vd = v_desc0 + static_cast<uint32_t>((stage * kTileBytes) >> 4);
    const uint32_t d = tmem + s * 256 + 128;
    const uint32_t a = tmem + s * 256;
    // P arrives in two halves (keys 0..63, 64..127); the first four K-steps start as soon as the
    // first half is in tensor memory.
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint32_t bar = ptx::smem_u32(half == 0 ? &sh.p_lo[s] : &sh.p_hi[s]);
      if (!wait_warp(bar, pr_phase[s], sh, p)) return false;
      ptx::tc_fence_after();
      if (leader) {
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int kk = half * 4 + k4;
          // V is [key][d] with d contiguous: MN-major B operand.  One K step = 16 keys = two
          // 8-row swizzle atoms (2 KB); the second 64-column half of d sits one TMA box later.
          ptx::mma_ts(d, a + kk * 8, vd + static_cast<uint32_t>((kk * 2048) >> 4), kIdescPV,
                      (x.j > 0 || kk > 0) ? 1u : 0u);
        }
      }
      __syncwarp();
    }
    pr_phase[s] ^= 1u;
    if (leader) {
      ptx::tc_commit(kv_empty0 + stage * 8);
      if (x.j == x.it.n_steps - 1) ptx::tc_commit(ptx::smem_u32(&sh.o_full[s]));
    }
    __syncwarp();
    if (++stage == kStages) stage = 0, kv_phase ^= 1u;
    return true;
  };

#pragma unroll
  for (int s = 0; s < 2; ++s) {
    st[s].g = 2 * blockIdx.x + s - 2 * gridDim.x;
    st[s].stride = 2 * gridDim.x;
    has[s] = next_active(st[s], p, nullptr);
    if (has[s] && ok) ok = issue_S(s);
  }
  while (ok && (has[0] || has[1])) {
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      if (!ok || !has[s]) continue;
      ok = issue_PV(s);
      if (!ok) continue;
      if (st[s].j + 1 < st[s].it.n_steps) {
        ++st[s].j;
        ok = issue_S(s);
      } else {
        has[s] = next_active(st[s], p, nullptr);
        if (has[s]) ok = issue_S(s);
      }
    }
  }
}

// ------------------------------------------------------------------------------------------
// Softmax + epilogue warpgroup for one slot.  Thread t owns query row t of the tile and the
// TMEM lane t (warp w of the group may only touch lanes 32*(w%4) .. +31).
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void store_row_f32(const FwdParams& p, size_t row, const float* v32,
                                              int col0, float mul, bool valid) {
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

__device__ void softmax_role(SharedStorage& sh, const FwdParams& p, int slot, uint32_t tmem) {
  const int t = threadIdx.x - slot * 128;
  const int wq = (threadIdx.x >> 5) & 3;
  const uint32_t lane_addr = tmem + (static_cast<uint32_t>(wq * 32) << 16);
  const uint32_t s_addr = lane_addr + slot * 256;
  const uint32_t o_addr = s_addr + 128;
  const uint32_t s_full = ptx::smem_u32(&sh.s_full[slot]);
  const uint32_t p_lo = ptx::smem_u32(&sh.p_lo[slot]);
  const uint32_t p_hi = ptx::smem_u32(&sh.p_hi[slot]);
  const uint32_t o_full = ptx::smem_u32(&sh.o_full[slot]);
  uint32_t sf_phase = 0, of_phase = 0;
  const float sl2 = p.scale_log2;

  for (int g = 2 * blockIdx.x + slot; g < p.total_items; g += 2 * gridDim.x) {
    const Item it = load_item(p, g, nullptr);
    const int q_pos = it.qb * kBlk + t;
    const size_t row = static_cast<size_t>(it.bh) * p.T + q_pos;
    if (it.n_steps == 0) {  // query block entirely past seq_len (v4 :63-68)
      float z[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) z[i] = 0.0f;
#pragma unroll
      for (int c = 0; c < 4; ++c) store_row_f32(p, row, z, c * 32, 0.0f, false);
      if (p.lse) p.lse[row] = -INFINITY;
      continue;
    }
    const bool row_valid = q_pos < it.seq_len;
    float m_run = -1e30f;  // v4 :74
    float l_run = 0.0f;

    for (int j = 0; j < it.n_steps; ++j) {
      bool ok = wait_bar(s_full, sf_phase, sh, p);
      if (!__all_sync(0xffffffffu, ok)) return;
      sf_phase ^= 1u;
      ptx::tc_fence_after();
      uint32_t sr[128];
      ptx::tmem_ld32(s_addr + 0, sr + 0);
      ptx::tmem_ld32(s_addr + 32, sr + 32);
      ptx::tmem_ld32(s_addr + 64, sr + 64);
      ptx::tmem_ld32(s_addr + 96, sr + 96);
      ptx::tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 128; ++c) ptx::reg_fence(sr[c]);
      float s[128];
#pragma unroll
      for (int c = 0; c < 128; ++c) s[c] = __uint_as_float(sr[c]);

      // Keys c >= n_keep are masked: the causal diagonal keeps c <= t (v4 :111; with t valid
      // that also keeps key < seq_len, v4 :112), an invalid query row keeps nothing (v4 :93).
      const bool diag = (j == it.n_steps - 1);
      const int n_keep = !row_valid ? 0 : (diag ? t + 1 : 128);
      if (n_keep < 128) {
#pragma unroll
        for (int c = 0; c < 128; ++c) s[c] = (c < n_keep) ? s[c] : -INFINITY;
      }
      // Row max of the raw scores (scale > 0 commutes with max), three inputs per instruction.
      float a0 = s[0], a1 = s[1], a2 = s[2], a3 = s[3];
#pragma unroll
      for (int c = 4; c < 124; c += 8) {
        a0 = ptx::fmax3(a0, s[c + 0], s[c + 1]);
        a1 = ptx::fmax3(a1, s[c + 2], s[c + 3]);
        a2 = ptx::fmax3(a2, s[c + 4], s[c + 5]);
        a3 = ptx::fmax3(a3, s[c + 6], s[c + 7]);
      }
      a0 = ptx::fmax3(a0, s[124], s[125]);
      a1 = ptx::fmax3(a1, s[126], s[127]);
      const float m_cand = ptx::fmax3(a0, a1, fmaxf(a2, a3)) * sl2;
      // Decide the new running max before touching O: P is computed against it, and O is
      // rescaled before the first half of P is released to the MMA.
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
      // p = 2^(s*scale - m) on pairs: one packed FMA per pair, MUFU for most exponentials and
      // the FMA-pipe polynomial for every kPolyEvery-th pair; the row sum l accumulates the
      // fp32 p (v4 :99) in packed adds; P is stored as fp16 pairs (v4 :103).
      const uint64_t sc2 = ptx::pack2(sl2, sl2);
      const uint64_t nm2 = ptx::pack2(-m_run, -m_run);
      uint64_t acc0 = 0, acc1 = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int c = 64 * h + 2 * i;
          const uint64_t x2 = ptx::ffma2(ptx::pack2(s[c], s[c + 1]), sc2, nm2);
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
        ptx::tmem_st32(s_addr + 32 * h, pk);
        if (h == 0 && rescale) {
          // O holds the sum through PV(j-1), which completed before S(j) was committed.
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
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
        ptx::mbar_arrive(h == 0 ? p_lo : p_hi);
      }
      float l0, l1, l2, l3;
      ptx::unpack2(ptx::fadd2(acc0, acc1), l0, l1);
      (void)l2;
      (void)l3;
      l_run += l0 + l1;
    }

    // Epilogue: o = O / l (v4 :126-133), lse = m ln2 + ln l (v4 :134-136).
    bool ok = wait_bar(o_full, of_phase, sh, p);
    if (!__all_sync(0xffffffffu, ok)) return;
    of_phase ^= 1u;
    ptx::tc_fence_after();
    const float inv_l = l_run > 0.0f ? 1.0f / l_run : 1.0f;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t orow[32];
      ptx::tmem_ld32(o_addr + c * 32, orow);
      ptx::tmem_wait_ld();
      float of[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        ptx::reg_fence(orow[i]);
        of[i] = __uint_as_float(orow[i]);
      }
      store_row_f32(p, row, of, c * 32, inv_l, row_valid);
    }
    if (p.lse) {
      const float lse = (row_valid && l_run > 0.0f) ? m_run * 0.69314718055994531f + logf(l_run)
                                                    : -INFINITY;
      p.lse[row] = lse;
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    bsattn_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                      const __grid_constant__ CUtensorMap tv, const __grid_constant__ FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = ptx::smem_u32(smem_raw);
  SharedStorage& sh =
      *reinterpret_cast<SharedStorage*>(smem_raw + (((raw + 1023u) & ~1023u) - raw));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(ptx::smem_u32(&sh.q_full[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&sh.q_empty[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&sh.s_full[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&sh.p_lo[s]), 128);
      ptx::mbar_init(ptx::smem_u32(&sh.p_hi[s]), 128);
      ptx::mbar_init(ptx::smem_u32(&sh.o_full[s]), 1);
    }
    for (int i = 0; i < kStages; ++i) {
      ptx::mbar_init(ptx::smem_u32(&sh.kv_full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&sh.kv_empty[i]), 1);
    }
    ptx::mbar_init(ptx::smem_u32(&sh.drain), 1);
    sh.abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kLoadWarp && lane == 0) {
    ptx::tma_prefetch_desc(&tq);
    ptx::tma_prefetch_desc(&tk);
    ptx::tma_prefetch_desc(&tv);
  }
  if (warp == kMmaWarp) {
    ptx::tmem_alloc(ptx::smem_u32(&sh.tmem_base), kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = sh.tmem_base;

  if (warp < 8) {
    ptx::setmaxnreg_inc<kSoftmaxRegs>();
    softmax_role(sh, p, warp >> 2, tmem);
  } else {
    ptx::setmaxnreg_dec<kControlRegs>();
    if (warp == kLoadWarp) {
      producer_role(sh, &tq, &tk, &tv, p, lane == 0);
    } else if (warp == kMmaWarp) {
      mma_role(sh, p, tmem, lane == 0);
    }
  }
  __syncwarp();
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    if (lane == 0) {
      // Every MMA this thread issued has completed once this commit arrives.
      ptx::tc_commit(ptx::smem_u32(&sh.drain));
      wait_drain(ptx::smem_u32(&sh.drain), 0, p);
    }
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

// [rows, 128] fp16 row-major, boxes of 128 rows x 64 columns, 128-byte swizzle.
static int make_tile_map(CUtensorMap* map, const void* base, uint64_t rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return BSATTN_E_TMA;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kHd), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(kHd * 2)};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kBlk)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides,
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

static size_t smem_bytes() { return sizeof(SharedStorage) + 1024; }

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
    if (fa.numRegs < static_cast<int>(kLaunchRegs) ||
        fa.numRegs * kThreads > 65536)
      return BSATTN_E_CUDA;
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

extern "C" {

size_t bsattn_workspace_bytes(void) { return kWsInts * sizeof(int); }

int bsattn_version(void) { return 100; }

void bsattn_set_timeout_ns(uint64_t ns) { g_timeout_ns = ns > 0 ? ns : 1; }

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
    case BSATTN_E_DTYPE: return "unsupported output dtype";
    default: return "unknown error";
  }
}

int bsattn_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
               const int32_t* row_ptr, const int32_t* col_idx, const int32_t* seq_lens, int B,
               int H, int T, int D, int64_t rp_stride_bh, int64_t ci_stride_bh, int max_nnz,
               float scale, int out_dtype, void* workspace, size_t workspace_bytes,
               void* stream) {
  if (!q || !k || !v || !o || !row_ptr || !col_idx) return BSATTN_E_NULL;
  if (B < 1 || H < 1 || T < kBlk || (T % kBlk) != 0 || D != kHd) return BSATTN_E_SHAPE;
  if (max_nnz < 0 || rp_stride_bh < 0 || ci_stride_bh < 0) return BSATTN_E_SHAPE;
  const long long rows = static_cast<long long>(B) * H * T;
  const long long items = static_cast<long long>(B) * H * (T / kBlk);
  if (rows >= (1ll << 31) || items >= (1ll << 30)) return BSATTN_E_SHAPE;
  if (out_dtype != BSATTN_OUT_F16 && out_dtype != BSATTN_OUT_BF16) return BSATTN_E_DTYPE;
  auto misaligned = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) != 0; };
  if (misaligned(q) || misaligned(k) || misaligned(v) || misaligned(o)) return BSATTN_E_ALIGN;
  if (!workspace || workspace_bytes < bsattn_workspace_bytes()) return BSATTN_E_WORKSPACE;

  int sms = 0;
  int rc = device_setup(&sms);
  if (rc != BSATTN_OK) return rc;

  CUtensorMap tq, tk, tv;
  if ((rc = make_tile_map(&tq, q, rows)) != BSATTN_OK) return rc;
  if ((rc = make_tile_map(&tk, k, rows)) != BSATTN_OK) return rc;
  if ((rc = make_tile_map(&tv, v, rows)) != BSATTN_OK) return rc;

  FwdParams p;
  memset(&p, 0, sizeof(p));
  p.row_ptr = row_ptr;
  p.col_idx = col_idx;
  p.seq_lens = seq_lens;
  p.o = o;
  p.lse = lse;
  p.ws = static_cast<int*>(workspace);
  p.rp_stride = rp_stride_bh;
  p.ci_stride = ci_stride_bh;
  p.max_nnz = max_nnz;
  p.BH = B * H;
  p.H = H;
  p.T = T;
  p.nqb = T / kBlk;
  p.total_items = static_cast<int>(items);
  const double sc = scale > 0.0f ? static_cast<double>(scale) : 1.0 / sqrt(static_cast<double>(D));
  p.scale_log2 = static_cast<float>(sc * 1.4426950408889634);
  p.out_bf16 = out_dtype == BSATTN_OUT_BF16 ? 1 : 0;
  p.timeout_ns = g_timeout_ns;

  const int grid = static_cast<int>(std::min<long long>(sms, (items + 1) / 2));
  bsattn_fwd_kernel<<<grid, kThreads, smem_bytes(), static_cast<cudaStream_t>(stream)>>>(tq, tk,
                                                                                        tv, p);
  return cudaGetLastError() == cudaSuccess ? BSATTN_OK : BSATTN_E_CUDA;
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
