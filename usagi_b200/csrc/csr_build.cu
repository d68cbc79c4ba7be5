// csr_build.cu -- CSR block patterns built on the device (the caller-side step before the
// attention call: row_ptr / col_idx over 128x128 blocks, one list per (batch, head)).
//
// Every row i lists its key blocks in ascending order and ends with its own diagonal i, the
// contract the reference kernel relies on (kernels/v4_leaderboard_0740ms.py:78-86, :107).
//   * window w / prefix p + window w: row i = {0 .. min(p-1, i)} U {max(0, i-w+1) .. i}.  A plain
//     window is p = 0.  Row lengths and offsets have closed forms, so one thread per (head, row)
//     writes its row_ptr entry and its columns with no scan; the result is bit-identical to the
//     host builder (usagi_b200/patterns.py).
//   * retrieval n: row i = {i-1, i} plus min(n, i-1) distinct blocks from 0 .. i-2, drawn
//     uniformly without replacement (Floyd's algorithm) from a counter-based SplitMix64 stream
//     keyed by (seed, head, row).  Same distribution as the host builder's randperm draws, not
//     the same draws: torch's CPU generator has no device counterpart.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/bsattn.h"

namespace bsattn_csr {

constexpr int kMaxRandom = 64;
// Largest prefix or window accepted (the same bound as the analytic rows of the attention entry
// point): prefix + window then stays far below INT_MAX, so the row arithmetic cannot wrap.
constexpr int kMaxWindow = 1 << 24;

struct Spec {
  int kind, nqb, prefix, window, n_random;
};

// row_ptr[i] = sum of the lengths of rows 0 .. i-1.  Row lengths: window / prefix+window rows
// hold i + 1 blocks while i < prefix + window and prefix + window after; retrieval rows hold
// i + 1 blocks for i < 2 and 2 + min(n_random, i - 1) after.
__host__ __device__ inline long long row_start(const Spec& s, long long i) {
  if (s.kind == BSATTN_CSR_RETRIEVAL) {
    if (i < 2) return i == 0 ? 0 : 1;
    const long long m = i - 2, n = s.n_random;
    const long long tri = m <= n ? m * (m + 1) / 2 : n * (n + 1) / 2 + (m - n) * n;
    return 3 + 2 * m + tri;
  }
  const long long L = static_cast<long long>(s.prefix) + s.window;
  return i <= L ? i * (i + 1) / 2 : L * (L + 1) / 2 + (i - L) * L;
}

__device__ inline uint64_t splitmix64(uint64_t& state) {
  uint64_t z = (state += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void __launch_bounds__(256) build_kernel(Spec s, uint64_t seed, int n_heads,
                                                    int32_t* __restrict__ row_ptr,
                                                    int32_t* __restrict__ col_idx,
                                                    long long ci_stride) {
  const long long idx = blockIdx.x * 256ll + threadIdx.x;
  if (idx >= static_cast<long long>(n_heads) * s.nqb) return;
  const int h = static_cast<int>(idx / s.nqb);
  const int i = static_cast<int>(idx - static_cast<long long>(h) * s.nqb);
  int32_t* rp = row_ptr + static_cast<long long>(h) * (s.nqb + 1);
  int32_t* out = col_idx + static_cast<long long>(h) * ci_stride + row_start(s, i);
  rp[i] = static_cast<int32_t>(row_start(s, i));
  if (i == s.nqb - 1) rp[s.nqb] = static_cast<int32_t>(row_start(s, s.nqb));

  if (s.kind != BSATTN_CSR_RETRIEVAL) {
    const long long L = static_cast<long long>(s.prefix) + s.window;
    if (i < L) {
      for (int c = 0; c <= i; ++c) out[c] = c;
    } else {
      for (int c = 0; c < s.prefix; ++c) out[c] = c;
      for (int c = 0; c < s.window; ++c) out[s.prefix + c] = i - s.window + 1 + c;
    }
    return;
  }
  if (i < 2) {
    for (int c = 0; c <= i; ++c) out[c] = c;
    return;
  }
  // Floyd: for j = N-r .. N-1 draw t in [0, j]; take t unless already taken, else take j.
  const int N = i - 1, r = min(s.n_random, N);
  int pick[kMaxRandom];
  uint64_t state = seed ^ (0xD1B54A32D192ED03ull * (static_cast<uint64_t>(h) * s.nqb + i + 1));
  for (int k = 0; k < r; ++k) {
    const int j = N - r + k;
    const uint32_t z = static_cast<uint32_t>(splitmix64(state) >> 32);
    int t = static_cast<int>((static_cast<uint64_t>(z) * static_cast<uint32_t>(j + 1)) >> 32);
    for (int u = 0; u < k; ++u)
      if (pick[u] == t) t = j;
    // Insertion keeps pick[0 .. k] sorted.
    int u = k;
    while (u > 0 && pick[u - 1] > t) {
      pick[u] = pick[u - 1];
      --u;
    }
    pick[u] = t;
  }
  for (int k = 0; k < r; ++k) out[k] = pick[k];
  out[r] = i - 1;
  out[r + 1] = i;
}

static int validate(const Spec& s) {
  if (s.kind < BSATTN_CSR_WINDOW || s.kind > BSATTN_CSR_RETRIEVAL) return BSATTN_E_SHAPE;
  if (s.nqb < 1 || s.nqb > (1 << 22)) return BSATTN_E_SHAPE;
  if (s.kind == BSATTN_CSR_RETRIEVAL) {
    if (s.n_random < 0 || s.n_random > kMaxRandom) return BSATTN_E_SHAPE;
  } else {
    if (s.window < 1 || s.prefix < 0 || s.window > kMaxWindow || s.prefix > kMaxWindow)
      return BSATTN_E_SHAPE;
    if (s.kind == BSATTN_CSR_WINDOW && s.prefix != 0) return BSATTN_E_SHAPE;
  }
  if (row_start(s, s.nqb) >= (1ll << 31)) return BSATTN_E_SHAPE;
  return BSATTN_OK;
}

}  // namespace bsattn_csr

extern "C" {

int bsattn_csr_nnz(int kind, int nqb, int prefix, int window, int n_random, int64_t* nnz) {
  const bsattn_csr::Spec s{kind, nqb, prefix, window, n_random};
  if (!nnz) return BSATTN_E_NULL;
  const int rc = bsattn_csr::validate(s);
  if (rc != BSATTN_OK) return rc;
  *nnz = bsattn_csr::row_start(s, nqb);
  return BSATTN_OK;
}

int bsattn_build_csr(int kind, int nqb, int prefix, int window, int n_random, uint64_t seed,
                     int n_heads, int32_t* row_ptr, int32_t* col_idx, int64_t ci_stride,
                     void* stream) {
  const bsattn_csr::Spec s{kind, nqb, prefix, window, n_random};
  if (!row_ptr || !col_idx) return BSATTN_E_NULL;
  int rc = bsattn_csr::validate(s);
  if (rc != BSATTN_OK) return rc;
  if (n_heads < 1 || ci_stride < bsattn_csr::row_start(s, nqb)) return BSATTN_E_SHAPE;
  const long long threads = static_cast<long long>(n_heads) * nqb;
  if (threads >= (1ll << 31)) return BSATTN_E_SHAPE;
  const unsigned grid = static_cast<unsigned>((threads + 255) / 256);
  bsattn_csr::build_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      s, seed, n_heads, row_ptr, col_idx, ci_stride);
  return cudaGetLastError() == cudaSuccess ? BSATTN_OK : BSATTN_E_CUDA;
}

}  // extern "C"
