// Token sampling on the GPU: temperature, top-k, top-p and a categorical draw
// for a batch of logit rows in one launch (vllm/sampler.py:7-42 of vllm-jax,
// which samples one request at a time with a device->host copy each).
//
// Semantics per row (reference line numbers in vllm/sampler.py):
//   temperature <= 0          argmax, first index on ties            (:12-14)
//   x = bf16(logit / T)       the reference divides the bf16 logits   (:16)
//   top_k > 0                 keep the top_k largest x; among equal
//                             values the lower index first (lax.top_k) (:17-23)
//   top_p < 1                 order the kept tokens by (x desc, index
//                             asc), keep those whose cumulative softmax
//                             probability is <= top_p; the first token is
//                             always kept                              (:25-36)
//   draw                      categorical over softmax(x) on the kept set
//                             by Gumbel-max, as jax.random.categorical (:38-41)
// Probabilities here are exact to 2^-32 (fixed-point sums, so the kept set is
// deterministic); the reference rounds softmax and cumsum to bf16. Random
// numbers come from Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel
// random numbers: as easy as 1, 2, 3", SC 2011) keyed by the row's 64-bit
// seed with counter (vocab index / 4, position, tag, 0), so a token depends
// only on (seed, position, logits), never on batch composition.
//
// One CTA per row, 512 threads, each owning 8 consecutive logits of a 4096-
// logit tile. Thresholds are found by radix selection over the 16-bit order
// key of the bf16 value x (two 256-bin histogram passes for top-k counts, two
// for top-p masses); a final pass ranks ties at the threshold by index with a
// block scan and takes the Gumbel argmax over the kept tokens. The row is
// re-read from L2 on every pass (a 152k-entry row is 304 KB).
#include "../../include/vjattn.h"
#include "vj_common.cuh"

#include <string>

namespace vj {
namespace {

constexpr int kSampThreads = 512;
constexpr int kPer = 8;
constexpr int kTile = kSampThreads * kPer;
constexpr int kWarps = kSampThreads / 32;
constexpr float kFix = 4294967296.0f;  // probabilities in 32.32 fixed point

// Order-preserving 16-bit key of a bf16 bit pattern (NaN -> 0, below all).
VJ_DEV uint32_t bf16_key(uint32_t b) {
  if ((b & 0x7F80u) == 0x7F80u && (b & 0x007Fu)) return 0u;
  return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
}
VJ_DEV float key_value(uint32_t k) {
  const uint32_t b = (k & 0x8000u) ? (k & 0x7FFFu) : (~k & 0xFFFFu);
  return __uint_as_float(b << 16);
}

// Philox4x32-10 block (SC 2011, section 3.3 / Random123 constants).
VJ_DEV void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c[0], hi0 = __umulhi(0xD2511F53u, c[0]);
    const uint32_t lo1 = 0xCD9E8D57u * c[2], hi1 = __umulhi(0xCD9E8D57u, c[2]);
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

// Gumbel noise from 32 random bits: u in (0, 1) on a 2^-23 grid.
VJ_DEV float gumbel(uint32_t r) {
  const float u = (static_cast<float>(r >> 9) + 0.5f) * 0x1p-23f;
  return -logf(-logf(u));
}

struct RowArgs {
  const __nv_bfloat16 *x;
  int vocab;
  float temp;
};

// Loads the 8 logits of this thread in tile `t`; returns how many are valid.
VJ_DEV int load8(const RowArgs &a, int t, uint32_t bits[kPer]) {
  const int base = t * kTile + threadIdx.x * kPer;
  if (base + kPer <= a.vocab) {
    const uint4 v = *reinterpret_cast<const uint4 *>(a.x + base);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      bits[2 * j] = w[j] & 0xFFFFu;
      bits[2 * j + 1] = w[j] >> 16;
    }
    return kPer;
  }
  int n = 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    if (base + j < a.vocab) {
      bits[j] = __bfloat16_as_ushort(a.x[base + j]);
      n = j + 1;
    } else {
      bits[j] = 0;
    }
  }
  return n;
}

// Keys of the temperature-scaled bf16 values x = bf16(logit / T).
VJ_DEV int load_keys(const RowArgs &a, int t, uint32_t key[kPer]) {
  uint32_t bits[kPer];
  const int n = load8(a, t, bits);
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const float l = __uint_as_float(bits[j] << 16);
    const uint32_t xb = __bfloat16_as_ushort(__float2bfloat16_rn(__fdiv_rn(l, a.temp)));
    key[j] = j < n ? bf16_key(xb) : 0u;
  }
  return n;
}

VJ_DEV uint64_t fixed_prob(uint32_t key, float xmax) {
  return __float2ull_rn(expf(key_value(key) - xmax) * kFix);
}

// Walk a 256-bin histogram from the top bin down. For counts, returns the
// first bin where (sum above + bin) >= target; for masses (strict), where
// (sum above + bin) > target. Run by one whole warp; result via shared memory.
template <typename T, bool kStrict>
VJ_DEV void find_cross(const T *hist, T target, int *bin_out, T *above_out, T *total_out) {
  const int lane = threadIdx.x & 31;
  // lane l owns bins 255-8l .. 248-8l (top first)
  T own[8];
  T s = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    own[j] = hist[255 - 8 * lane - j];
    s += own[j];
  }
  T incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  const T total = __shfl_sync(0xffffffffu, incl, 31);
  T above = incl - s;
  int found = -1;
  T found_above = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const bool hit = kStrict ? (above + own[j] > target) : (above + own[j] >= target);
    if (found < 0 && hit) {
      found = 255 - 8 * lane - j;
      found_above = above;
    }
    above += own[j];
  }
  const unsigned m = __ballot_sync(0xffffffffu, found >= 0);
  if (lane == 0) {
    *total_out = total;
    *bin_out = -1;
    *above_out = total;
  }
  __syncwarp();
  if (m) {
    const int src = __ffs(m) - 1;
    const int b = __shfl_sync(0xffffffffu, found, src);
    const T ab = __shfl_sync(0xffffffffu, found_above, src);
    if (lane == 0) {
      *bin_out = b;
      *above_out = ab;
    }
  }
}

struct SampleShared {
  uint32_t cnt[256];
  unsigned long long mass[256];
  uint32_t red_u[kWarps];
  float red_f[kWarps];
  int red_i[kWarps];
  uint32_t scan[kWarps];
  int bin;
  uint32_t above_cnt, total_cnt;
  unsigned long long above_mass, total_mass;
};

__global__ void __launch_bounds__(kSampThreads)
sample_kernel(const __nv_bfloat16 *__restrict__ logits, int64_t row_stride, int vocab,
              const float *__restrict__ temperature, const int32_t *__restrict__ top_k,
              const float *__restrict__ top_p, const uint32_t *__restrict__ seeds,
              int32_t *out_tokens, int32_t *num_kept, int32_t *token_table, int token_stride,
              const int32_t *seq_slots, const int32_t *seq_lens) {
  __shared__ SampleShared sh;
  const int row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  RowArgs a{logits + (size_t)row * row_stride, vocab, temperature[row]};
  const int ntiles = (vocab + kTile - 1) / kTile;
  int token = 0, kept = 1;

  if (!(a.temp > 0.f)) {
    // ---- greedy: argmax of the raw logits, NaN first, lowest index on ties
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int t = 0; t < ntiles; ++t) {
      uint32_t bits[kPer];
      const int n = load8(a, t, bits);
      const int base = t * kTile + tid * kPer;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        if (j < n) {
          float v = __uint_as_float(bits[j] << 16);
          if (v != v) v = INFINITY;
          if (v > best) { best = v; idx = base + j; }
        }
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
    }
    if (lane == 0) { sh.red_f[warp] = best; sh.red_i[warp] = idx; }
    __syncthreads();
    if (warp == 0) {
      best = lane < kWarps ? sh.red_f[lane] : -INFINITY;
      idx = lane < kWarps ? sh.red_i[lane] : 0x7fffffff;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
      }
      if (lane == 0) sh.red_i[0] = idx == 0x7fffffff ? 0 : idx;
    }
    __syncthreads();
    token = sh.red_i[0];
  } else {
    // ---- pass 1: largest key
    uint32_t kmax = 0;
    for (int t = 0; t < ntiles; ++t) {
      uint32_t key[kPer];
      load_keys(a, t, key);
#pragma unroll
      for (int j = 0; j < kPer; ++j) kmax = max(kmax, key[j]);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
    if (lane == 0) sh.red_u[warp] = kmax;
    __syncthreads();
    if (warp == 0) {
      uint32_t v = lane < kWarps ? sh.red_u[lane] : 0u;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
      if (lane == 0) sh.red_u[0] = v;
    }
    __syncthreads();
    kmax = sh.red_u[0];
    const float xmax = key_value(kmax);

    // threshold: keys > thr kept; keys == thr kept for the first `lim` by index
    int thr = -1;
    uint32_t lim = 0xffffffffu;
    uint32_t n_above = 0;  // kept tokens with key > thr (valid when thr >= 0)
    const int k = top_k[row];
    if (k > 0 && k < vocab) {
      // ---- passes 2-3: top-k by counts
      for (int i = tid; i < 256; i += kSampThreads) sh.cnt[i] = 0;
      __syncthreads();
      for (int t = 0; t < ntiles; ++t) {
        uint32_t key[kPer];
        const int n = load_keys(a, t, key);
#pragma unroll
        for (int j = 0; j < kPer; ++j) if (j < n) atomicAdd(&sh.cnt[key[j] >> 8], 1u);
      }
      __syncthreads();
      if (warp == 0) find_cross<uint32_t, false>(sh.cnt, (uint32_t)k, &sh.bin, &sh.above_cnt,
                                                  &sh.total_cnt);
      __syncthreads();
      const int hb = sh.bin;
      const uint32_t above_hi = sh.above_cnt;
      __syncthreads();
      for (int i = tid; i < 256; i += kSampThreads) sh.cnt[i] = 0;
      __syncthreads();
      for (int t = 0; t < ntiles; ++t) {
        uint32_t key[kPer];
        const int n = load_keys(a, t, key);
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
          if (j < n && (int)(key[j] >> 8) == hb) atomicAdd(&sh.cnt[key[j] & 0xFFu], 1u);
        }
      }
      __syncthreads();
      if (warp == 0) find_cross<uint32_t, false>(sh.cnt, (uint32_t)k - above_hi, &sh.bin,
                                                  &sh.above_cnt, &sh.total_cnt);
      __syncthreads();
      thr = (hb << 8) | sh.bin;
      n_above = above_hi + sh.above_cnt;
      const uint32_t ties = sh.cnt[sh.bin];
      lim = min((uint32_t)k - n_above, ties);
      __syncthreads();
    }
    const float p = top_p[row];
    if (p < 1.0f) {
      // ---- passes 4-5: top-p by fixed-point probability mass over the kept set
      const uint64_t tie_q = thr >= 0 ? fixed_prob((uint32_t)thr, xmax) : 0ull;
      for (int i = tid; i < 256; i += kSampThreads) { sh.cnt[i] = 0; sh.mass[i] = 0ull; }
      __syncthreads();
      for (int t = 0; t < ntiles; ++t) {
        uint32_t key[kPer];
        const int n = load_keys(a, t, key);
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
          if (j < n && (int)key[j] > thr) {
            atomicAdd(&sh.mass[key[j] >> 8], (unsigned long long)fixed_prob(key[j], xmax));
            atomicAdd(&sh.cnt[key[j] >> 8], 1u);
          }
        }
      }
      __syncthreads();
      if (tid == 0 && thr >= 0) {
        sh.mass[thr >> 8] += (unsigned long long)lim * tie_q;
        sh.cnt[thr >> 8] += lim;
      }
      __syncthreads();
      // total mass first (target unknown yet): a crossing search with target max
      if (warp == 0) {
        find_cross<unsigned long long, true>(sh.mass, ~0ull, &sh.bin, &sh.above_mass,
                                             &sh.total_mass);
      }
      __syncthreads();
      const unsigned long long Z = sh.total_mass;
      const unsigned long long P =
          (unsigned long long)floor((double)p * (double)Z);
      __syncthreads();
      if (warp == 0) {
        find_cross<unsigned long long, true>(sh.mass, P, &sh.bin, &sh.above_mass,
                                             &sh.total_mass);
        // count of kept tokens in bins above the crossing one
        uint32_t c = 0;
        const int b = sh.bin;
        for (int i = lane; i < 256; i += 32) if (i > b) c += sh.cnt[i];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
        if (lane == 0) sh.above_cnt = c;
      }
      __syncthreads();
      const int hb = sh.bin;
      if (hb >= 0) {  // otherwise every kept token stays (no crossing)
        const unsigned long long above_hi = sh.above_mass;
        const uint32_t above_hi_cnt = sh.above_cnt;
        __syncthreads();
        for (int i = tid; i < 256; i += kSampThreads) { sh.cnt[i] = 0; sh.mass[i] = 0ull; }
        __syncthreads();
        for (int t = 0; t < ntiles; ++t) {
          uint32_t key[kPer];
          const int n = load_keys(a, t, key);
#pragma unroll
          for (int j = 0; j < kPer; ++j) {
            if (j < n && (int)key[j] > thr && (int)(key[j] >> 8) == hb) {
              atomicAdd(&sh.mass[key[j] & 0xFFu], (unsigned long long)fixed_prob(key[j], xmax));
              atomicAdd(&sh.cnt[key[j] & 0xFFu], 1u);
            }
          }
        }
        __syncthreads();
        if (tid == 0 && thr >= 0 && (thr >> 8) == hb) {
          sh.mass[thr & 0xFF] += (unsigned long long)lim * tie_q;
          sh.cnt[thr & 0xFF] += lim;
        }
        __syncthreads();
        if (warp == 0) {
          find_cross<unsigned long long, true>(sh.mass, P - above_hi, &sh.bin, &sh.above_mass,
                                               &sh.total_mass);
          uint32_t c = 0;
          const int b = sh.bin;
          for (int i = lane; i < 256; i += 32) if (i > b) c += sh.cnt[i];
#pragma unroll
          for (int o = 16; o >= 1; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
          if (lane == 0) sh.above_cnt = c;
        }
        __syncthreads();
        const int tp = (hb << 8) | sh.bin;
        const unsigned long long m_above = above_hi + sh.above_mass;
        const uint32_t n_tp = sh.cnt[sh.bin];
        const uint64_t e_tp = fixed_prob((uint32_t)tp, xmax);
        uint64_t room = P - m_above;  // P >= m_above by the crossing rule
        uint64_t l = e_tp ? room / e_tp : (uint64_t)n_tp;
        if (l > n_tp) l = n_tp;
        n_above = above_hi_cnt + sh.above_cnt;
        if (n_above == 0 && l == 0) l = 1;  // the first token is always kept
        thr = tp;
        lim = (uint32_t)l;
        __syncthreads();
      }
    }
    kept = thr < 0 ? vocab : (int)(n_above + lim);

    // ---- pass 6: Gumbel argmax over the kept tokens; ties at thr ranked by index
    const uint32_t s0 = seeds[2 * row], s1 = seeds[2 * row + 1];
    const uint32_t pos = seq_lens ? (uint32_t)seq_lens[row] : 0u;
    float best = -INFINITY;
    int idx = 0x7fffffff;
    uint32_t tie_base = 0;  // ties at thr in earlier tiles
    for (int t = 0; t < ntiles; ++t) {
      uint32_t key[kPer];
      const int n = load_keys(a, t, key);
      uint32_t my_ties = 0;
#pragma unroll
      for (int j = 0; j < kPer; ++j) my_ties += (j < n && (int)key[j] == thr) ? 1u : 0u;
      uint32_t rank = 0;
      if (__syncthreads_or(my_ties != 0)) {
        uint32_t incl = my_ties;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += v;
        }
        if (lane == 31) sh.scan[warp] = incl;
        __syncthreads();
        uint32_t wbase = 0, tile_total = 0;
        for (int w = 0; w < kWarps; ++w) {
          const uint32_t v = sh.scan[w];
          if (w < warp) wbase += v;
          tile_total += v;
        }
        rank = tie_base + wbase + incl - my_ties;
        tie_base += tile_total;
        __syncthreads();
      }
      const int base = t * kTile + tid * kPer;
      bool any = false;
      bool keep[kPer];
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        bool kj = j < n && (int)key[j] >= thr;
        if (kj && (int)key[j] == thr) {
          kj = rank < lim;
          ++rank;
        }
        keep[j] = kj;
        any |= kj;
      }
      if (any) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t c[4] = {(uint32_t)(base / 4 + h), pos, 0x53414D50u, 0u};
          philox4x32_10(c, s0, s1);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int j = 4 * h + q;
            if (keep[j]) {
              const float sc = key_value(key[j]) + gumbel(c[q]);
              if (sc > best) { best = sc; idx = base + j; }
            }
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
    }
    if (lane == 0) { sh.red_f[warp] = best; sh.red_i[warp] = idx; }
    __syncthreads();
    if (warp == 0) {
      best = lane < kWarps ? sh.red_f[lane] : -INFINITY;
      idx = lane < kWarps ? sh.red_i[lane] : 0x7fffffff;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
      }
      if (lane == 0) sh.red_i[0] = idx == 0x7fffffff ? 0 : idx;
    }
    __syncthreads();
    token = sh.red_i[0];
  }
  if (tid == 0) {
    out_tokens[row] = token;
    if (num_kept) num_kept[row] = kept;
    if (token_table && seq_slots && seq_lens) {
      const int slot = seq_slots[row], len = seq_lens[row];
      if (slot >= 0 && len >= 0 && len < token_stride) {
        token_table[(size_t)slot * token_stride + len] = token;
      }
    }
  }
}

}  // namespace
}  // namespace vj

extern "C" vj_status vj_sample(const void *logits, int64_t row_stride, int32_t num_rows,
                               int32_t vocab, const float *temperature, const int32_t *top_k,
                               const float *top_p, const uint32_t *seeds, int32_t *out_tokens,
                               int32_t *num_kept, int32_t *token_table, int32_t token_stride,
                               const int32_t *seq_slots, const int32_t *seq_lens,
                               cudaStream_t stream) {
  using namespace vj;
  if (num_rows < 0 || vocab <= 0 || row_stride < vocab) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_sample: bad sizes");
  }
  if (num_rows == 0) return VJ_OK;
  if (!logits || !temperature || !top_k || !top_p || !seeds || !out_tokens) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_sample: null pointer");
  }
  if (token_table && (!seq_slots || !seq_lens)) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_sample: token_table needs seq_slots/seq_lens");
  }
  if ((reinterpret_cast<uintptr_t>(logits) & 15u) || (row_stride & 7)) {
    return set_error(VJ_ERR_UNSUPPORTED,
                     "vj_sample: logits must be 16-byte aligned with a row stride multiple of 8");
  }
  sample_kernel<<<num_rows, kSampThreads, 0, stream>>>(
      static_cast<const __nv_bfloat16 *>(logits), row_stride, vocab, temperature, top_k, top_p,
      seeds, out_tokens, num_kept, token_table, token_stride, seq_slots, seq_lens);
  return check_launch("vj_sample");
}
