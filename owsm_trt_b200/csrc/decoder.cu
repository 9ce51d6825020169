// The OWSM decoder call as one persistent kernel for sm_100a, and the C ABI around it (include/owsm_dec.h).
//
// Semantics: owsm-trt's Decoder.step (src/owsm_trt/modeling.py:501-560) with the megakernel's in-kernel
// cache write (src/owsm_trt/megakernel.py:321-326), fused argmax (src/owsm_trt/megakernel_ring.py:437-500)
// and BeamSession._select step 1 + cache reorder (src/owsm_trt/runtime.py:1399-1413).
//
// Execution model (one CTA per SM, all co-resident: cooperative launch):
//   * warp 8 of every CTA is the producer: lane 0 walks the CTA's whole sequence of input byte ranges for
//     the call (its GEMM weight row blocks, the KV-cache rows of its self-attention units, the encoder K/V
//     frames of its cross-attention pieces) and copies them with cp.async.bulk into a ring of 32 KB
//     shared-memory slots, running ahead of the computation across the stage boundaries, so HBM streams
//     while the CTAs wait for each other.
//   * warps 0-7 consume the slots stage by stage; between stages a bounded grid barrier.
//   * stages: embedding; per layer LN1+QKV, self-attention, out-proj+residual, LN2+cross-Q,
//     cross-attention, cross-out+residual, LN3+FFN1+ReLU, FFN2+residual; final LN + vocabulary projection
//     (+ argmax or per-CTA log-softmax / top-K partials); for beam calls: selection, cache reorder (2 stages).
//   * GEMMs: y[token, n] = sum_k W[n, k] x[token, k] with mma.sync m16n8k16 (fp16 in, fp32 accumulate),
//     weights as the 16-row A operand, prepacked in fragment order so each lane loads 16 contiguous bytes;
//     LayerNorm folded into the weights (W*gamma, b + W beta) and the normalised activations computed by
//     every CTA that needs them from the fp32 residual stream.
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/owsm_dec.h"
#include "ptx.cuh"

namespace owsm {

constexpr int DK = 64;                 // head size (every OWSM model)
constexpr int XPS = DK + 4;            // floats per query of a cross-attention partial: 64 outputs, max, sum, 2 pad
constexpr int NWARP = 7;               // consumer warps (+1 producer: 8 warps, 2 per SM sub-partition)
constexpr int NTHR = NWARP * 32;       // consumer threads
constexpr int BLOCK = NTHR + 32;       // + producer warp
constexpr int SLOT = 32768;            // ring slot bytes
constexpr int MAXSLOT = 8;
constexpr int MAXNT = 8;               // n-tiles of 8 tokens: M <= 64 tokens per call
constexpr int MAXQ = 32;               // queries of one attention unit (grid-stage kernel)
constexpr int CLQ = 16;                // queries of one attention unit (cluster kernel)
constexpr int KTOP = 8;                // largest beam
constexpr int APOS = SLOT / (DK * 2);  // attention positions per chunk (256)
constexpr uint32_t DEFAULT_SPIN = 1u << 22;

enum Gemm { G_QKV = 0, G_WO, G_CQ, G_WCO, G_F1, G_F2, G_OUT, NGEMM };
enum { E_ERR_TIMEOUT = 1 };

struct GemmW {
  const uint4* w;   // packed fragments: [layer][block][kblock][lane] of 16 bytes
  const float* b;   // [layer][N]
  int N, K, NB;     // output rows, input features, 16-row blocks
  long long lstride;  // uint4 elements per layer
  int bstride;        // uint4 elements per 16-row block: K/16 k-blocks x 32 lanes + the block's 16 fp32 biases
};

struct PlanDev {
  int L, D, H, F, V, max_pos;
  float eps, xscale;
  int R, S, M, NT, C, T, G, U, beam, P, nslot;
  int slot, apos;  // ring slot bytes, attention positions per chunk (slot / 128)
  int sstride;     // bytes between slots: slot + room for a block's 64-byte bias tail
  uint32_t max_spin;
  const __half* emb;
  const float* pe;
  GemmW g[NGEMM];
  const int* goff[NGEMM];  // [P + 1]
  const int* gblk[NGEMM];
  float* x;       // [M][D] residual stream
  __half* qkv;    // [M][3D]
  __half* q2;     // [M][D]
  __half* oB;     // attention outputs, B-fragment order [D/16][NT][32][4]
  __half* hB;     // FFN hidden, B-fragment order [F/16][NT][32][4]
  float* xpart;   // cross-attention partials [U*H][P][Q][XPS]
  uint32_t* xcnt; // [U*H]
  float* amax;    // [P][M]
  int* aidx;      // [P][M]
  float* lmax;    // [P][M]
  float* lsum;    // [P][M]
  int* cstart;    // [R] beam calls: the first cache slot a row takes from its parent (shared prefixes known)
  float* topv;    // [P][M][KTOP]
  int* topi;      // [P][M][KTOP]
  uint32_t* ctr;  // [0] grid barrier, [1] exits, [2] argmax arrivals
  int* err;
  int Qmax;           // queries of the largest attention unit
  unsigned long long* ts;  // optional stamps [stage][P][4] (profiling), NULL = off
  int ev_from;              // profiling: the stage from which CTAs log events (0: from the start)
  int off_pre, off_out, off_ring, off_work;  // shared-memory layout (bytes)
  int off_sched, off_rows;  // this CTA's block lists and the rows' cache offsets (shared memory)
  int inflight;             // bulk copies in flight per CTA (ring slots may hold more, finished)
  int stage_b;              // largest non-LayerNorm B operand staged in shared memory (bytes)
  int work_bytes;           // size of the work area
  const long long* xfix;    // cluster kernel: the fixed-point residual stream the output stage normalises
  int cl;                   // 1: the cluster kernel runs this plan
  int RG, NCL3, F3;         // cluster kernel: row groups per head, clusters of the FFN stage, hidden units each
  int wide;                 // cluster kernel: one-query attention units of >= 256 positions take steps of 32
  int Rs, Us;               // cluster kernel: rows / utterances of the caller's buffers (layer strides of the
                            // caches, new_kv and cross K/V), more than R / U when the call is a row slice
  int kvg;                  // cluster kernel, beam calls: attention groups (one row each) per copy of cross K/V
                            // and per enc_len entry (the utterance's hypotheses); 0 or 1 = one each
  long long* xf[3];         // cluster kernel: rotating fixed-point residual buffers [M][D]
  // dense kernel (calls of 33 to 64 tokens; tcgen05 GEMMs)
  int dense;
  const __half* gt[NGEMM];  // weights in 128-row tiles [layer][tile][K / 64][128 x 64] (canonical K-major)
  long long gtl[NGEMM];     // halves per layer
  int nsplit[NGEMM];        // K ranges per tile
  float* part;              // partial sums of split tiles [tile][range][64 tokens][128 rows]
  uint32_t* tcnt;           // ranges arrived per tile (the last one resets it)
  __half* obuf;             // attention output in the token-operand layout [D / 8][8][64] halves
  __half* hbuf;             // FFN hidden in the token-operand layout [F / 8][8][64] halves
  float* xstat;             // LayerNorm partial sums of the residual rows [D / 128][64 tokens][sum, sum of squares]
  const float* gcs[NGEMM];  // row sums of the LayerNorm-folded fp16 weights [layer][N] (the GEMMs after a LayerNorm)
  __half* xop;              // the residual rows as the token operand: fp16 high parts [D / 64 blocks][64][64], then
                            // the low parts (x - high) in the same layout
  int off_stat;             // shared memory: the stage's LayerNorm mean and 1 / std per token [64][2]
};

struct CallArgs {
  const int64_t* tok;
  int64_t tok_stride;
  const int64_t* off;
  int64_t off_stride;
  __half* kc;
  __half* vc;
  const __half* ck;
  const __half* cv;
  const int32_t* enc_len;
  float* logits;
  __half* new_kv;
  int64_t* pred;
  const uint8_t* notime;
  int ft, lt;
  // verify calls: the input rows, timestamp rules (ESPnet's ScoreFilter) on the argmax, the drafted tokens accepted
  const int64_t* inp;  // [R] rows of [S tokens | offset | timestamps so far | last timestamp | first position]
  int64_t inp_stride;
  int rules;           // 1: the argmax under the timestamp rules (ft, lt, eos; notime = the rows' flags)
  int eos;
  int64_t* res;        // [R][2]: drafted tokens accepted, the argmax after them (NULL: not wanted)
  float* score;
  const uint8_t* active;
  int64_t* parent;
  int64_t* token;
  int32_t* shared;  // beam calls, NULL or [R / beam][beam][beam]: cache slots each pair of rows holds in common
  int beam_mode;
};

// ------------------------------------------------------------------------------------------------ helpers
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(NTHR) : "memory"); }

__device__ __forceinline__ void mma16816(float (&c)[4], const uint4& a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

__device__ __forceinline__ int row_off_global(const PlanDev& pd, const CallArgs& a, int r) {
  long long o = a.off[(long long)r * a.off_stride];
  long long hi = pd.C - pd.S;
  return (int)(o < 0 ? 0 : (o > hi ? hi : o));
}

// Per-CTA facts staged in shared memory at kernel start, so no stage waits on a global load for them
// (under full weight streaming an L2 round trip costs microseconds): the CTA's 16-row blocks per GEMM
// (so[gi] .. so[gi + 1] index sb) and every row's clamped cache offset.
struct Ctx {
  const int* so;
  const int* sb;
  const int* offs;
  unsigned long long* ev;  // profiling: event stamps of this CTA (thread 0), NULL = off
  int* nev;                // shared-memory event counter
  float* red;              // [2 * NWARP] shared-memory partial sums of a LayerNorm team
};

constexpr int NEV = 128;  // events per CTA in the profiling log
__device__ __forceinline__ void event(const Ctx& cx, int tag) {
  if (cx.ev && threadIdx.x == 0 && *cx.nev < NEV - 1) {
    long long clk;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(clk));
    cx.ev[*cx.nev] = globaltimer();
    cx.ev[*cx.nev + 1] = ((unsigned long long)clk << 8) | (unsigned)tag;
    *cx.nev += 2;
  }
}

// The copy of cross K/V (and its enc_len entry) that attention group u reads.
__device__ __forceinline__ int kv_utt(const PlanDev& pd, int u) { return pd.kvg > 1 ? u / pd.kvg : u; }

__device__ __forceinline__ int utt_len(const PlanDev& pd, const CallArgs& a, int u) {
  int t = a.enc_len ? a.enc_len[kv_utt(pd, u)] : pd.T;
  return t < 1 ? 1 : (t > pd.T ? pd.T : t);
}

// Half index of element (token m, feature k) in B-fragment order with NT n-tiles (32-bit: every B operand,
// in shared or global memory, holds far fewer than 2^31 halves).
__device__ __forceinline__ int bfrag_idx(int m, int k, int NT) {
  const int kb = k >> 4, kk = k & 15, nt = m >> 3, g = m & 7;
  const int reg = kk >> 3, t = (kk & 7) >> 1, e = kk & 1;
  return (((kb * NT + nt) * 32 + (g * 4 + t)) * 4) + reg * 2 + e;
}

// The frame-space partition of cross-attention: frames of all (utterance, head) segments in a row,
// split in P contiguous ranges (P = min(CTAs, frames), so no range is empty).
struct Frames {
  long long total;
  int U, H, P;
  const int* pre;  // [U + 1] prefix sums of utterance lengths (shared memory)
  __device__ long long bound(int c) const { return c >= P ? total : (long long)c * total / P; }
  // The CTA whose range holds frame f: the largest c with floor(c * total / P) <= f, i.e. c * total <
  // (f + 1) * P, i.e. c = ceil((f + 1) * P / total) - 1 (one division, no search).
  __device__ int owner(long long f) const {
    const long long c = ((f + 1) * P + total - 1) / total - 1;
    return (int)(c < P - 1 ? c : P - 1);
  }
  __device__ int utt_of(long long f) const {  // utterance of flat frame f
    int lo = 0, hi = U - 1;
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if ((long long)H * pre[mid] <= f) lo = mid; else hi = mid - 1;
    }
    return lo;
  }
};

// One piece of a CTA's cross-attention range: segment (u, h) frames [t0, t1).
struct Piece {
  int u, h, t0, t1;
};

__device__ __forceinline__ bool next_piece(const Frames& fr, long long& f, long long end, Piece& p) {
  if (f >= end) return false;
  int u = fr.utt_of(f);
  int len = fr.pre[u + 1] - fr.pre[u];
  long long base = (long long)fr.H * fr.pre[u];
  int h = (int)((f - base) / len);
  int t0 = (int)(f - base - (long long)h * len);
  long long t1 = t0 + (end - f);
  if (t1 > len) t1 = len;
  p.u = u; p.h = h; p.t0 = t0; p.t1 = (int)t1;
  f += t1 - t0;
  return true;
}

// ------------------------------------------------------------------------------------------------ stages
// Stage index g: 0 embed; 1 + 8 l + i for i in (QKV, SATT, WO, CQ, XATT, WCO, F1, F2); 8 L + 1 output;
// beam calls: 8 L + 2 select, 8 L + 3 reorder A, 8 L + 4 reorder B.
enum Kind { K_EMBED, K_QKV, K_SATT, K_WO, K_CQ, K_XATT, K_WCO, K_F1, K_F2, K_OUT, K_SELECT, K_REORDER };

__device__ __forceinline__ Kind stage_kind(const PlanDev& pd, int g, int& layer) {
  layer = 0;
  if (g == 0) return K_EMBED;
  if (g <= 8 * pd.L) {
    layer = (g - 1) >> 3;
    return (Kind)(K_QKV + ((g - 1) & 7));
  }
  int i = g - 8 * pd.L - 1;
  return (Kind)(K_OUT + i);
}

__device__ __forceinline__ int gemm_of(Kind k) {
  switch (k) {
    case K_QKV: return G_QKV;
    case K_WO: return G_WO;
    case K_CQ: return G_CQ;
    case K_WCO: return G_WCO;
    case K_F1: return G_F1;
    case K_F2: return G_F2;
    case K_OUT: return G_OUT;
    default: return -1;
  }
}

// Chunk enumeration shared by the producer (issues the copies) and the consumer (waits for them):
// calls f(src, bytes) for every chunk of stage g on CTA c, in consumption order.
template <class Fn>
__device__ void for_chunks(const PlanDev& pd, const CallArgs& a, const Frames& fr, const Ctx& cx, int g, int c,
                           Fn&& f) {
  int layer;
  Kind k = stage_kind(pd, g, layer);
  int gi = gemm_of(k);
  if (gi >= 0) {
    const GemmW gw = pd.g[gi];
    int l = (k == K_OUT) ? 0 : layer;
    int kbs = gw.K >> 4;
    int kpc = kbs < (pd.slot / 512) ? kbs : (pd.slot / 512);  // k-blocks per chunk
    for (int i = cx.so[gi]; i < cx.so[gi + 1]; ++i) {
      int rb = cx.sb[i];
      const uint4* base = gw.w + (long long)l * gw.lstride + (long long)rb * gw.bstride;
      for (int kb0 = 0; kb0 < kbs; kb0 += kpc) {
        int n = kbs - kb0 < kpc ? kbs - kb0 : kpc;
        // the block's biases (64 bytes) come with its last chunk
        f((const void*)(base + (long long)kb0 * 32), (uint32_t)n * 512 + (kb0 + n == kbs ? 64u : 0u));
      }
    }
    return;
  }
  if (k == K_SATT) {
    for (int u = c; u < pd.R * pd.H; u += pd.P) {
      int b = u / pd.H, h = u % pd.H;
      int off = cx.offs[b];
      long long base = ((((long long)layer * pd.R + b) * pd.H + h) * pd.C) * DK;
      for (int j0 = 0; j0 < off; j0 += pd.apos) {
        int n = off - j0 < pd.apos ? off - j0 : pd.apos;
        f((const void*)(a.kc + base + (long long)j0 * DK), (uint32_t)n * DK * 2);
        f((const void*)(a.vc + base + (long long)j0 * DK), (uint32_t)n * DK * 2);
      }
    }
    return;
  }
  if (k == K_XATT) {
    long long f0 = fr.bound(c), f1 = fr.bound(c + 1);
    Piece p;
    while (next_piece(fr, f0, f1, p)) {
      long long base = ((((long long)layer * pd.U + p.u) * pd.H + p.h) * pd.T) * DK;
      for (int j0 = p.t0; j0 < p.t1; j0 += pd.apos) {
        int n = p.t1 - j0 < pd.apos ? p.t1 - j0 : pd.apos;
        f((const void*)(a.ck + base + (long long)j0 * DK), (uint32_t)n * DK * 2);
        f((const void*)(a.cv + base + (long long)j0 * DK), (uint32_t)n * DK * 2);
      }
    }
  }
}

struct Ring {
  uint64_t* full;
  uint64_t* empty;
  uint8_t* data;
  int ns, stride;
  uint32_t i;     // chunks consumed so far
  uint32_t spin;
  int* err;
  bool dead;
  unsigned long long waited;  // ns spent waiting for slots (thread 0, when tracing)
  bool timing;
  __device__ uint8_t* wait() {
    int s = i % ns;
    unsigned long long t0 = timing ? globaltimer() : 0;
    if (!dead && !mbar_wait(&full[s], (i / ns) & 1, spin)) {
      dead = true;
      atomicExch(err, E_ERR_TIMEOUT);
    }
    if (timing) waited += globaltimer() - t0;
    return data + (size_t)s * stride;
  }
  __device__ void release() {  // by every consumer warp after its last read of the slot
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&empty[i % ns]);
    ++i;
  }
  // One warp alone consumes chunk `idx` (its arrival counts for all the consumer warps).
  __device__ uint8_t* wait_at(uint32_t idx) {
    const int s = idx % ns;
    unsigned long long t0 = timing ? globaltimer() : 0;
    if (!dead && !mbar_wait(&full[s], (idx / ns) & 1, spin)) {
      dead = true;
      atomicExch(err, E_ERR_TIMEOUT);
    }
    if (timing) waited += globaltimer() - t0;
    return data + (size_t)s * stride;
  }
  __device__ void release_at(uint32_t idx, int cnt = NWARP) {  // cnt: this warp's share of the NWARP arrivals
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive_cnt(&empty[idx % ns], cnt);
  }
};

// Grid barrier: all P CTAs arrive after their stage; bounded wait; the counter resets at kernel exit.
// sdead (shared memory, optional): thread 0 publishes there whether the call has failed (its own timed-out
// wait or any CTA's error word), and every consumer thread takes it over as `dead`.
__device__ void grid_sync(const PlanDev& pd, uint32_t target, bool& dead, int* sdead = nullptr) {
  csync();
  if (threadIdx.x == 0) {
    red_release_add(&pd.ctr[0], 1);
    if (!dead && !*(volatile int*)pd.err) {
      uint32_t n = 0;
      while ((int)(ld_acquire(&pd.ctr[0]) - target) < 0) {
        if (++n > pd.max_spin) {
          atomicExch(pd.err, E_ERR_TIMEOUT);
          dead = true;
          break;
        }
      }
    }
    // any CTA's failure: its error word was set before its arrival, so after the acquiring poll it is visible
    if (*(volatile int*)pd.err) dead = true;
    if (sdead) *sdead = dead ? 1 : 0;
  }
  csync();
  if (sdead) dead = *sdead != 0;
}

// ------------------------------------------------------------------------------------------------ GEMM
struct Work {  // shared-memory work area, carved per stage
  uint8_t* p;
};

// LayerNorm of the residual stream x [M][D] (eps) into B-fragment order (fp16) in shared memory. One warp
// per token; a lane holds its D / 32 values in registers (all loads issued at once: one L2 round trip).
constexpr int MAXV4 = 8;  // D <= 1024: float4 loads per lane
// Four consecutive values of a residual-stream row: fp32, or int64 fixed point (32 fraction bits).
__device__ __forceinline__ float4 load4(const float* row, int i) { return __ldcg(reinterpret_cast<const float4*>(row) + i); }
__device__ __forceinline__ float4 load4(const long long* row, int i) {
  const longlong2 a = __ldcg(reinterpret_cast<const longlong2*>(row) + 2 * i);
  const longlong2 b = __ldcg(reinterpret_cast<const longlong2*>(row) + 2 * i + 1);
  return make_float4(from_fix(a.x), from_fix(a.y), from_fix(b.x), from_fix(b.y));
}

// Zero fragments for the padding tokens M .. NT * 8 - 1 of a B operand over D features.
__device__ __forceinline__ void zero_pad_tokens(__half* bbuf, int M, int NT, int D) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int m = M + warp; m < NT * 8; m += NWARP)
    for (int k = lane * 2; k < D; k += 64) *reinterpret_cast<uint32_t*>(&bbuf[bfrag_idx(m, k, NT)]) = 0u;
}

// LayerNorm of rows m0 .. m0 + M - 1 of the residual stream into the B operand (fragment order over NT
// tiles of 8 tokens, shared memory), padding tokens zero.
// From 7 rows on, a warp normalises whole rows; below that a row is split over a team of 7 / M warps whose
// partial sums meet in shared memory, so one row costs one round trip for its loads and a few hundred
// cycles rather than a single warp's serial pass over 1024 values.
// r0 .. r1 - 1 (default: all M) are the tokens this call normalises; the padding is zeroed either way.
// pad = false: the caller keeps the padding tokens' fragments zero itself.
template <class T>
__device__ void ln_rows(const PlanDev& pd, const T* x, int m0, int M, int NT, __half* bbuf, const Ctx& cx,
                        int r0 = 0, int r1 = -1, bool pad = true) {
  const int D = pd.D, nv = D / 4;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  event(cx, 21);
  if (pad) zero_pad_tokens(bbuf, M, NT, D);
  event(cx, 22);
  if (r1 < 0) r1 = M;
  const int Mc = r1 - r0;
  const int ts = Mc >= NWARP ? 1 : NWARP / Mc;  // warps per row
  auto emit = [&](int m, int i, const float4& v, float mean, float rstd) {
    const int k = i * 4;
    *reinterpret_cast<__half2*>(&bbuf[bfrag_idx(m, k, NT)]) =
        __floats2half2_rn((v.x - mean) * rstd, (v.y - mean) * rstd);
    *reinterpret_cast<__half2*>(&bbuf[bfrag_idx(m, k + 2, NT)]) =
        __floats2half2_rn((v.z - mean) * rstd, (v.w - mean) * rstd);
  };
  // One pass of statistics: the sum and the sum of squares in fp64 (a float's square is exact in double,
  // so E[x^2] - mean^2 keeps full fp32 accuracy), one shuffle round and, for a team, one barrier.
  auto moments = [&](const float4& u, double& s1, double& s2) {
    s1 += ((double)u.x + (double)u.y) + ((double)u.z + (double)u.w);
    s2 = fma((double)u.x, (double)u.x, s2);
    s2 = fma((double)u.y, (double)u.y, s2);
    s2 = fma((double)u.z, (double)u.z, s2);
    s2 = fma((double)u.w, (double)u.w, s2);
  };
  auto finish = [&](double s1, double s2, float& mean, float& rstd) {
    const double mu = s1 / D, var = fmax(s2 / D - mu * mu, 0.0);
    mean = (float)mu;
    rstd = rsqrtf((float)var + pd.eps);
  };
  if (ts == 1) {
    for (int m = r0 + warp; m < r1; m += NWARP) {
      const T* xr = x + (long long)(m0 + m) * D;
      float4 v[MAXV4];
#pragma unroll
      for (int i = 0; i < MAXV4; ++i)
        if (i * 32 + lane < nv) v[i] = load4(xr, i * 32 + lane);
      double s1 = 0.0, s2 = 0.0;
#pragma unroll
      for (int i = 0; i < MAXV4; ++i)
        if (i * 32 + lane < nv) moments(v[i], s1, s2);
      event(cx, 20);
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        s1 += __shfl_xor_sync(0xffffffffu, s1, o);
        s2 += __shfl_xor_sync(0xffffffffu, s2, o);
      }
      float mean, rstd;
      finish(s1, s2, mean, rstd);
#pragma unroll
      for (int i = 0; i < MAXV4; ++i)
        if (i * 32 + lane < nv) emit(m, i * 32 + lane, v[i], mean, rstd);
    }
    return;
  }
  // teams: row m = warp / ts (warps past M * ts only join the barrier); member j takes float4s
  // j * 32 + lane + k * ts * 32; the members' sums meet in shared memory (cx.red as 2 x NWARP doubles)
  const int mt = warp / ts, m = r0 + mt, j = warp % ts, step = ts * 32;
  const bool on = mt < Mc;
  double* red = reinterpret_cast<double*>(cx.red);
  float4 v[MAXV4];
  if (on) {
    const T* xr = x + (long long)(m0 + m) * D;
#pragma unroll
    for (int k = 0; k < MAXV4; ++k)
      if (j * 32 + lane + k * step < nv) v[k] = load4(xr, j * 32 + lane + k * step);
    double s1 = 0.0, s2 = 0.0;
#pragma unroll
    for (int k = 0; k < MAXV4; ++k)
      if (j * 32 + lane + k * step < nv) moments(v[k], s1, s2);
    event(cx, 20);
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    if (lane == 0) {
      red[warp] = s1;
      red[NWARP + warp] = s2;
    }
  }
  csync();
  event(cx, 23);
  if (on) {
    double s1 = 0.0, s2 = 0.0;
    for (int w = mt * ts; w < mt * ts + ts; ++w) {
      s1 += red[w];
      s2 += red[NWARP + w];
    }
    float mean, rstd;
    finish(s1, s2, mean, rstd);
#pragma unroll
    for (int k = 0; k < MAXV4; ++k)
      if (j * 32 + lane + k * step < nv) emit(m, j * 32 + lane + k * step, v[k], mean, rstd);
  }
}

// The B operand of a LayerNorm GEMM stage over all M tokens: from the fp32 residual stream, or from the
// fixed-point one of the cluster kernel when the plan names it.
__device__ void ln_to_frag(const PlanDev& pd, __half* bbuf, const Ctx& cx) {
  if (pd.xfix) ln_rows(pd, pd.xfix, 0, pd.M, pd.NT, bbuf, cx);
  else ln_rows(pd, pd.x, 0, pd.M, pd.NT, bbuf, cx);
}

// Per-token running results of the output stage (shared memory). The CTA-level arrays hold the stage's
// result; the per-warp arrays the warps' running state while they multiply their own blocks.
struct OutState {
  float* amax;  // [M] argmax (greedy)
  int* aidx;
  float* rmax;  // [M] log-softmax partials and top-K (beam)
  float* rsum;
  float* topv;  // [M][KTOP]
  int* topi;
  float* wamax;  // [NWARP][M]
  int* waidx;
  float* wrmax;  // [NWARP][M] (beam)
  float* wrsum;
  float* wtopv;  // [NWARP][M][KTOP]
  int* wtopi;
  float* wtile;  // [NWARP][16][M]
};

// Timestamp rules of the argmax (runtime.py:457-492 TimestampRules.forbidden, applied per window position as
// _Verify.predict, runtime.py:1251-1267): the state of token m = (row r, position i) from its input row --
// timestamps so far (count, last) plus those the window adds at positions 1 .. i, the token at i, whether i is
// the first generated position, the row's <notimestamps> flag -- packed into st[0] (bits: no-time, first, odd
// count, previous token a timestamp) and st[1] (last timestamp).
__device__ __forceinline__ void rule_state(const PlanDev& pd, const CallArgs& a, int m, int* st) {
  const int W = pd.S, r = m / W, i = m - r * W;
  const int64_t* row = a.inp + (long long)r * a.inp_stride;
  long long count = row[W + 1], last = row[W + 2];
  for (int j = 1; j <= i; ++j) {
    const long long t = row[j];
    if (t >= a.ft && t <= a.lt) {
      ++count;
      last = t > last ? t : last;
    }
  }
  const long long prev = row[i];
  const int flags = (a.notime && a.notime[r] ? 1 : 0) | (row[W + 3] == i ? 2 : 0) | ((count & 1) ? 4 : 0) |
                    ((prev >= a.ft && prev <= a.lt) ? 8 : 0);
  st[0] = flags;
  st[1] = (int)(last < -1 ? -1 : (last > 0x7fffffff ? 0x7fffffff : last));
}

// Whether id v is forbidden for a token in state st (rule_state).
__device__ __forceinline__ bool rule_bad(const int* st, int v, const CallArgs& a) {
  const int f = st[0], last = st[1];
  const bool time = v >= a.ft && v <= a.lt;
  if (f & 1) return time;
  if (f & 2) return !time;
  if (f & 4) return v == a.eos || (time && v <= last);
  if (f & 8) return (v < last || v > a.lt) && v != a.eos;
  return true;
}

// Forbidden for the argmax of token m: the full rules when the call has them, else the <notimestamps> mask.
__device__ __forceinline__ bool argmax_bad(const PlanDev& pd, const CallArgs& a, const int* st, int m, int n) {
  if (a.rules) return rule_bad(st, n, a);
  return a.notime && n >= a.ft && n <= a.lt && a.notime[m / pd.S];
}

// Candidate order of the beam select: value descending, then flat index ascending.
__device__ __forceinline__ bool beats(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

__device__ __forceinline__ void merge_best(float& bv, int& bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

// Output stage, beam calls: the 16 values of a block (tile[16][M], this warp's) into the warp's running
// log-sum-exp and top-K per token; lane m handles token m (and m + 32).
__device__ __forceinline__ void beam_merge_block(OutState& os, int warp, int lane, int M, int rb) {
  const float* tile = os.wtile + (size_t)warp * 16 * M;
  for (int m = lane; m < M; m += 32) {
    float* rm = os.wrmax + warp * M + m;
    float* rs = os.wrsum + warp * M + m;
    float bmx = *rm;
    for (int row = 0; row < 16; ++row) bmx = fmaxf(bmx, tile[row * M + m]);
    if (bmx > -INFINITY) {
      float sm = (*rm > -INFINITY) ? *rs * expf(*rm - bmx) : 0.f;
      for (int row = 0; row < 16; ++row) {
        const float y = tile[row * M + m];
        if (y > -INFINITY) sm += expf(y - bmx);
      }
      *rm = bmx;
      *rs = sm;
    }
    float* tv = os.wtopv + ((size_t)warp * M + m) * KTOP;
    int* ti = os.wtopi + ((size_t)warp * M + m) * KTOP;
    for (int row = 0; row < 16; ++row) {
      const float y = tile[row * M + m];
      const int n = rb * 16 + row;
      if (!(y > tv[KTOP - 1] || (y == tv[KTOP - 1] && n < ti[KTOP - 1]))) continue;
      int j = KTOP - 1;
      while (j > 0 && (y > tv[j - 1] || (y == tv[j - 1] && n < ti[j - 1]))) {
        tv[j] = tv[j - 1];
        ti[j] = ti[j - 1];
        --j;
      }
      tv[j] = y;
      ti[j] = n;
    }
  }
}

// Epilogue of one 16-row block from a warp's accumulators: lane (g, t) owns rows g, g + 8 and tokens
// 2t, 2t + 1 of every n-tile. bia = the block's biases of rows g, g + 8; xres = residual inputs (prefetched).
template <int NT>
__device__ __forceinline__ void block_epilogue(const PlanDev& pd, const CallArgs& a, Kind kind, int rb,
                                               const float (&acc)[NT][4], const float (&bia)[2],
                                               const float (&xres)[NT][4], float (&best)[NT][2],
                                               int (&besti)[NT][2], OutState& os, int warp, int lane) {
  const int M = pd.M, D = pd.D, V = pd.V, N = pd.g[gemm_of(kind)].N;
  const int g = lane >> 2, t = lane & 3;
  if (kind == K_OUT && a.beam_mode) {
    float* tile = os.wtile + (size_t)warp * 16 * M;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = g + (e >> 1) * 8, m = nt * 8 + 2 * t + (e & 1), n = rb * 16 + row;
        if (m < M) {
          const float y = acc[nt][e] + bia[e >> 1];
          if (n < V) a.logits[(long long)m * V + n] = y;
          tile[row * M + m] = (n < V) ? y : -INFINITY;
        }
      }
    __syncwarp();
    beam_merge_block(os, warp, lane, M, rb);
    __syncwarp();
    return;
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = g + (e >> 1) * 8, m = nt * 8 + 2 * t + (e & 1), n = rb * 16 + row;
      if (m >= M || n >= N) continue;
      const float y = acc[nt][e] + bia[e >> 1];
      switch (kind) {
        case K_QKV: pd.qkv[(long long)m * 3 * D + n] = __float2half_rn(y); break;
        case K_CQ: pd.q2[(long long)m * D + n] = __float2half_rn(y); break;
        case K_F1: pd.hB[bfrag_idx(m, n, NT)] = __float2half_rn(fmaxf(y, 0.f)); break;
        case K_WO: case K_WCO: case K_F2: pd.x[(long long)m * D + n] = xres[nt][e] + y; break;
        case K_OUT: {
          a.logits[(long long)m * V + n] = y;
          float ya = y;
          if (argmax_bad(pd, a, os.topi + m * KTOP, m, n)) ya = -INFINITY;
          merge_best(best[nt][e & 1], besti[nt][e & 1], ya, n);
          break;
        }
        default: break;
      }
    }
}

__device__ void combine_cross_to_frag(const PlanDev& pd, const Frames& fr, __half* bbuf, float* stage, int cap,
                                      int* offs_s, const Ctx& cx);

// One GEMM stage on this CTA. Work items are the ring chunks of the CTA's 16-row blocks (a chunk: 16 rows x
// up to 64 k-blocks); warp w multiplies chunks w, w + 7, ... from start to end (two accumulator chains,
// pointer-increment addressing), and writes the block's outputs from its registers. Blocks longer than one
// chunk (FFN2 at K = 4096) leave per-chunk partial sums in shared memory, added up in chunk order after the
// stage. The B operand (activations) is in shared memory: LayerNorm stages normalise x there; the others
// copy the attention output / FFN hidden there once per stage when it fits, else read it from L2.
template <int NT>
__device__ void gemm_stage(const PlanDev& pd, const CallArgs& a, Ring& ring, const Ctx& cx, const Frames& fr,
                           Kind kind, int layer, int c, uint8_t* work, OutState& os) {
  const int gi = gemm_of(kind);
  const GemmW gw = pd.g[gi];
  const int nb0 = cx.so[gi], nb1 = cx.so[gi + 1];
  if (nb0 == nb1) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  event(cx, 9);
  const int M = pd.M, D = pd.D;
  const bool ln = (kind == K_QKV || kind == K_CQ || kind == K_F1 || kind == K_OUT);
  const bool res = (kind == K_WO || kind == K_WCO || kind == K_F2);
  const int l = (kind == K_OUT) ? 0 : layer;
  const int kbs = gw.K >> 4;
  const int kpc = kbs < (pd.slot / 512) ? kbs : (pd.slot / 512);
  const int cpu = (kbs + kpc - 1) / kpc;  // chunks per block
  const int nb = nb1 - nb0, nch = nb * cpu;
  __half* bbuf = reinterpret_cast<__half*>(work);
  const size_t bbytes = (size_t)NT * kbs * 256;
  const bool staged = ln || kind == K_WO || kind == K_WCO || bbytes <= (size_t)pd.stage_b;
  float* red = reinterpret_cast<float*>(work + (staged ? bbytes : 0));  // [nch][NT][32][4] + [nb][16] biases
  float* redb = red + (size_t)nch * NT * 128;
  const uint2* gsrc = reinterpret_cast<const uint2*>((kind == K_F2) ? pd.hB : pd.oB);
  const int g = lane >> 2, t = lane & 3;
  const int ns = ring.ns;
  const int j0 = warp < ns ? (warp - (int)(ring.i % (uint32_t)ns) + ns) % ns : nch;
  // residual inputs of this warp's first block, in flight together with the B operand's loads
  float xfirst[NT][4];
  if (res) {
    const int u0 = (cpu == 1) ? j0 : warp;  // multi-chunk blocks: the block this warp finishes first
    const bool have = (cpu == 1) ? (j0 < nch) : (warp < nb);
    const int rb0 = have ? cx.sb[nb0 + u0] : 0;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int m = nt * 8 + 2 * t + (e & 1), nn = rb0 * 16 + g + (e >> 1) * 8;
        xfirst[nt][e] = (have && m < M && nn < gw.N) ? __ldcg(pd.x + (long long)m * D + nn) : 0.f;
      }
  }
  if (ln) {
    ln_to_frag(pd, bbuf, cx);
  } else if (kind == K_WCO) {  // combine the cross-attention partials into the B operand
    // staging area: the work area after the B operand, minus a small table of segment offsets
    int* segoff = reinterpret_cast<int*>(work + pd.work_bytes) - (pd.U * pd.H + 1 + NWARP + 4);
    float* stage = reinterpret_cast<float*>(work + bbytes);
    const int cap = (int)((reinterpret_cast<uint8_t*>(segoff) - reinterpret_cast<uint8_t*>(stage)) / 4) - 64;
    combine_cross_to_frag(pd, fr, bbuf, stage, cap, segoff, cx);
  } else if (staged) {  // the whole B operand of the stage into shared memory: one L2 round trip
    const uint4* src = reinterpret_cast<const uint4*>(gsrc);
    uint4* dst = reinterpret_cast<uint4*>(bbuf);
    const int n16 = (int)(bbytes / 16);
#pragma unroll 4
    for (int i = threadIdx.x; i < n16; i += NTHR) dst[i] = __ldcg(src + i);
  }
  event(cx, 10 + kind);
  if (kind == K_OUT && a.rules && !a.beam_mode)  // the timestamp-rule state of every token (greedy calls)
    for (int m = threadIdx.x; m < M; m += NTHR) rule_state(pd, a, m, os.topi + m * KTOP);
  if (kind == K_OUT) {  // this warp's running output state
    for (int m = lane; m < M; m += 32) {
      os.wamax[warp * M + m] = -INFINITY;
      os.waidx[warp * M + m] = 0x7fffffff;
      if (a.beam_mode) {
        os.wrmax[warp * M + m] = -INFINITY;
        os.wrsum[warp * M + m] = 0.f;
        for (int j = 0; j < KTOP; ++j) {
          os.wtopv[((size_t)warp * M + m) * KTOP + j] = -INFINITY;
          os.wtopi[((size_t)warp * M + m) * KTOP + j] = 0x7fffffff;
        }
      }
    }
  }
  csync();
  event(cx, 30);
  float best[NT][2];
  int besti[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) best[nt][0] = best[nt][1] = -INFINITY, besti[nt][0] = besti[nt][1] = 0x7fffffff;
  const uint32_t bsh = smem_u32(bbuf);
  // Warp w takes the chunks that land in ring slot w (warps beyond the slot count idle here): each slot is
  // consumed by one warp in order, so no waiter is ever two phases ahead of a slot's barrier (a parity wait
  // cannot tell phases two apart).
  for (int j = j0; j < nch; j += ns) {
    const int u = j / cpu, part = j - u * cpu;
    const int rb = cx.sb[nb0 + u];
    const int kb0 = part * kpc;
    const int n = kbs - kb0 < kpc ? kbs - kb0 : kpc;
    const bool last = (part == cpu - 1);
    float xres[NT][4];
    if (res && cpu == 1) {  // residual inputs of this block (the first block's were loaded with the B operand)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int m = nt * 8 + 2 * t + (e & 1), nn = rb * 16 + g + (e >> 1) * 8;
          xres[nt][e] = (j == j0) ? xfirst[nt][e] : ((m < M && nn < gw.N) ? __ldcg(pd.x + (long long)m * D + nn) : 0.f);
        }
    }
    const uint8_t* slot = ring.wait_at(ring.i + j);
    event(cx, 31);
    const uint32_t ash = smem_u32(slot) + lane * 16;
    float acc0[NT][4], acc1[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc0[nt][e] = acc1[nt][e] = 0.f;
    if (staged) {
      uint32_t bp = bsh + ((uint32_t)kb0 * NT * 32 + lane) * 8;
#pragma unroll 2
      for (int kb = 0; kb < n; kb += 2) {
        const uint4 a0 = lds128_u32(ash + kb * 512);
        const uint4 a1 = lds128_u32(ash + (kb + 1) * 512);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint2 b0 = lds64_u32(bp + nt * 256);
          const uint2 b1 = lds64_u32(bp + (NT + nt) * 256);
          mma16816(acc0[nt], a0, b0.x, b0.y);
          mma16816(acc1[nt], a1, b1.x, b1.y);
        }
        bp += 2 * NT * 256;
      }
    } else {
      const uint2* bg = gsrc + ((long long)kb0 * NT) * 32 + lane;
#pragma unroll 2
      for (int kb = 0; kb < n; kb += 2) {
        const uint4 a0 = lds128_u32(ash + kb * 512);
        const uint4 a1 = lds128_u32(ash + (kb + 1) * 512);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint2 b0 = __ldcg(bg + nt * 32);
          const uint2 b1 = __ldcg(bg + (NT + nt) * 32);
          mma16816(acc0[nt], a0, b0.x, b0.y);
          mma16816(acc1[nt], a1, b1.x, b1.y);
        }
        bg += 2 * NT * 32;
      }
    }
    float bia[2] = {0.f, 0.f};
    if (last) {  // the block's biases (rows g, g + 8) from the chunk's tail
      const float* tail = reinterpret_cast<const float*>(slot + (size_t)n * 512);
      bia[0] = tail[g];
      bia[1] = tail[g + 8];
    }
    ring.release_at(ring.i + j);
    event(cx, 32);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc0[nt][e] += acc1[nt][e];
    if (cpu == 1) {
      block_epilogue<NT>(pd, a, kind, rb, acc0, bia, xres, best, besti, os, warp, lane);
    } else {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        sts128f(&red[(((size_t)j * NT + nt) * 32 + lane) * 4],
                make_float4(acc0[nt][0], acc0[nt][1], acc0[nt][2], acc0[nt][3]));
      if (last && t == 0) {
        redb[u * 16 + g] = bia[0];
        redb[u * 16 + g + 8] = bia[1];
      }
    }
  }
  event(cx, 33);
  ring.i += nch;
  if (cpu > 1) {  // blocks of several chunks: their partial sums in chunk order
    csync();
    for (int u = warp; u < nb; u += NWARP) {
      const int rb = cx.sb[nb0 + u];
      float acc[NT][4], xres[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int m = nt * 8 + 2 * t + (e & 1), nn = rb * 16 + g + (e >> 1) * 8;
          xres[nt][e] = (u == warp) ? xfirst[nt][e]
                                    : ((res && m < M && nn < gw.N) ? __ldcg(pd.x + (long long)m * D + nn) : 0.f);
          acc[nt][e] = 0.f;
        }
      for (int part = 0; part < cpu; ++part) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float4 q = lds128f(&red[((((size_t)u * cpu + part) * NT + nt) * 32 + lane) * 4]);
          acc[nt][0] += q.x; acc[nt][1] += q.y; acc[nt][2] += q.z; acc[nt][3] += q.w;
        }
      }
      const float bia[2] = {redb[u * 16 + g], redb[u * 16 + g + 8]};
      block_epilogue<NT>(pd, a, kind, rb, acc, bia, xres, best, besti, os, warp, lane);
    }
  }
  if (kind == K_OUT && !a.beam_mode) {  // the warp's best per token (over its row groups), then over the warps
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int s2 = 0; s2 < 2; ++s2) {
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, best[nt][s2], o);
          const int oi = __shfl_xor_sync(0xffffffffu, besti[nt][s2], o);
          merge_best(best[nt][s2], besti[nt][s2], ov, oi);
        }
        const int m = nt * 8 + 2 * t + s2;
        if (g == 0 && m < M) {
          os.wamax[warp * M + m] = best[nt][s2];
          os.waidx[warp * M + m] = besti[nt][s2];
        }
      }
  }
  csync();
  if (kind == K_OUT) {  // per-CTA results from the warps' states
    for (int m = threadIdx.x; m < M; m += NTHR) {
      if (!a.beam_mode) {
        float bv = os.amax[m];
        int bi = os.aidx[m];
        for (int w = 0; w < NWARP; ++w) merge_best(bv, bi, os.wamax[w * M + m], os.waidx[w * M + m]);
        os.amax[m] = bv;
        os.aidx[m] = bi;
      } else {
        float mx = os.rmax[m];
        for (int w = 0; w < NWARP; ++w) mx = fmaxf(mx, os.wrmax[w * M + m]);
        float sm = (os.rmax[m] > -INFINITY) ? os.rsum[m] * expf(os.rmax[m] - mx) : 0.f;
        for (int w = 0; w < NWARP; ++w) {
          const float wm = os.wrmax[w * M + m];
          if (wm > -INFINITY) sm += os.wrsum[w * M + m] * expf(wm - mx);
        }
        os.rmax[m] = mx;
        os.rsum[m] = sm;
        float* tv = os.topv + m * KTOP;
        int* ti = os.topi + m * KTOP;
        for (int w = 0; w < NWARP; ++w)
          for (int e = 0; e < KTOP; ++e) {
            const float y = os.wtopv[((size_t)w * M + m) * KTOP + e];
            const int n = os.wtopi[((size_t)w * M + m) * KTOP + e];
            if (!(y > tv[KTOP - 1] || (y == tv[KTOP - 1] && n < ti[KTOP - 1]))) continue;
            int jj = KTOP - 1;
            while (jj > 0 && (y > tv[jj - 1] || (y == tv[jj - 1] && n < ti[jj - 1]))) {
              tv[jj] = tv[jj - 1];
              ti[jj] = ti[jj - 1];
              --jj;
            }
            tv[jj] = y;
            ti[jj] = n;
          }
      }
    }
    csync();
  }
}

// ------------------------------------------------------------------------------------------------ attention
// Online-softmax attention of Q queries (q_s [Q][64], scaled) over chunks of keys/values; each warp keeps
// partial outputs for positions j = warp (mod NWARP) in registers: lane owns dims 2*lane, 2*lane + 1.
// QM = compile-time bound of Q (1: single-query units, the greedy decode step).
template <int QM>
struct AttnAcc {
  float o[QM][2];
};

// scores[q][j] = q . K[j] for j < npos (K rows in shared memory, 128 bytes each), several queries:
// a thread per (query, position).
__device__ __forceinline__ void attn_scores_multi(const float* qs, const __half* kt, int npos, int Q, float* sc) {
  for (int idx = threadIdx.x; idx < Q * npos; idx += NTHR) {
    const int q = idx / npos, j = idx - q * npos;
    const uint4* kr = reinterpret_cast<const uint4*>(kt + (long long)j * DK);
    const float* qq = qs + q * DK;
    float s = 0.f;
#pragma unroll
    for (int cc = 0; cc < 8; ++cc) {
      const int ch = (cc + j) & 7;  // rotate the 16-byte chunk per position: fewer bank conflicts
      const uint4 kv = kr[ch];
      const __half2* h2 = reinterpret_cast<const __half2*>(&kv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(h2[e]);
        s += f.x * qq[ch * 8 + 2 * e] + f.y * qq[ch * 8 + 2 * e + 1];
      }
    }
    sc[q * APOS + j] = s;
  }
}

// One query: four lanes per position (16 dims each, the query's 16 dims in registers), eight positions per
// warp per step; each lane's quarter of the row is rotated by its position group so the eight rows of a
// step fall in different banks.
struct Q1Regs {
  float q[16];
  int part;
};

__device__ __forceinline__ Q1Regs q1_load(const float* qs) {
  Q1Regs r;
  const int lane = threadIdx.x & 31;
  r.part = ((lane & 3) + (lane >> 2)) & 3;
#pragma unroll
  for (int i = 0; i < 16; ++i) r.q[i] = qs[r.part * 16 + i];
  return r;
}

__device__ __forceinline__ void attn_scores_q1(const Q1Regs& qr, const __half* kt, int npos, float* sc) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = smem_u32(kt) + qr.part * 32;
  for (int j0 = warp * 8; j0 < npos; j0 += NWARP * 8) {
    const int j = j0 + (lane >> 2);
    float s = 0.f;
    if (j < npos) {
      const uint4 k0 = lds128_u32(base + j * 128);
      const uint4 k1 = lds128_u32(base + j * 128 + 16);
      const __half2* h0 = reinterpret_cast<const __half2*>(&k0);
      const __half2* h1 = reinterpret_cast<const __half2*>(&k1);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f0 = __half22float2(h0[e]);
        const float2 f1 = __half22float2(h1[e]);
        s += f0.x * qr.q[2 * e] + f0.y * qr.q[2 * e + 1] + f1.x * qr.q[8 + 2 * e] + f1.y * qr.q[9 + 2 * e];
      }
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if ((lane & 3) == 0 && j < npos) sc[j] = s;
  }
}

// Softmax bookkeeping of a chunk: new running max per query, p = exp(s - max) in place, alpha (rescale of
// the old sums), running sum. `valid(q, j)` masks positions.
template <class Valid>
__device__ __forceinline__ void attn_softmax(float* sc, int npos, int Q, float* mrun, float* lrun, float* alpha,
                                             Valid valid) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int q = warp; q < Q; q += NWARP) {
    float mx = -INFINITY;
    for (int j = lane; j < npos; j += 32)
      if (valid(q, j)) mx = fmaxf(mx, sc[q * APOS + j]);
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float mold = mrun[q];
    const float mnew = fmaxf(mold, mx);
    float sum = 0.f;
    for (int j = lane; j < npos; j += 32) {
      const float p = (valid(q, j) && mnew > -INFINITY) ? expf(sc[q * APOS + j] - mnew) : 0.f;
      sc[q * APOS + j] = p;
      sum += p;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
      const float al = (mold > -INFINITY) ? expf(mold - mnew) : 0.f;
      alpha[q] = al;
      lrun[q] = lrun[q] * al + sum;
      mrun[q] = mnew;
    }
  }
}

template <int QM>
__device__ __forceinline__ void attn_accum(AttnAcc<QM>& acc, const float* sc, const float* alpha, const __half* vt,
                                           int npos, int Q) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int q = 0; q < QM; ++q)
    if (q < Q) {
      acc.o[q][0] *= alpha[q];
      acc.o[q][1] *= alpha[q];
    }
  const uint32_t vb = smem_u32(vt) + lane * 4;
  for (int j = warp; j < npos; j += NWARP) {
    uint32_t raw;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(raw) : "r"(vb + j * 128));
    const float2 v = __half22float2(*reinterpret_cast<__half2*>(&raw));
#pragma unroll
    for (int q = 0; q < QM; ++q)
      if (q < Q) {
        const float p = sc[q * APOS + j];
        acc.o[q][0] += p * v.x;
        acc.o[q][1] += p * v.y;
      }
  }
}

// Sum the warps' partial outputs into out[q][64] (shared memory).
template <int QM>
__device__ __forceinline__ void attn_reduce(const AttnAcc<QM>& acc, int Q, float* scratch, float* out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int q = 0; q < QM; ++q)
    if (q < Q) {
      scratch[(warp * Q + q) * DK + 2 * lane] = acc.o[q][0];
      scratch[(warp * Q + q) * DK + 2 * lane + 1] = acc.o[q][1];
    }
  csync();
  for (int idx = threadIdx.x; idx < Q * DK; idx += NTHR) {
    const int q = idx / DK, d = idx % DK;
    float s = 0.f;
    for (int w = 0; w < NWARP; ++w) s += scratch[(w * Q + q) * DK + d];
    out[q * DK + d] = s;
  }
  csync();
}

struct AttnSmem {
  float* q;      // [Q][64]
  float* sc;     // [Q][APOS]
  float* mrun;   // [MAXQ]
  float* lrun;
  float* alpha;
  float* knew;   // [Q][64] (self-attention: the new keys, fp32)
  float* vnew;   // [Q][64] (self-attention: the new values, fp32)
  float* out;    // [Q][64]
  float* scratch;  // [NWARP][Q][64]
  int* flag;
};

__device__ AttnSmem carve_attn(uint8_t* work, int Q) {
  AttnSmem s;
  float* p = reinterpret_cast<float*>(work);
  s.q = p; p += Q * DK;
  s.sc = p; p += Q * APOS;
  s.mrun = p; p += MAXQ;
  s.lrun = p; p += MAXQ;
  s.alpha = p; p += MAXQ;
  s.knew = p; p += Q * DK;
  s.vnew = p; p += Q * DK;
  s.out = p; p += Q * DK;
  s.scratch = p; p += NWARP * Q * DK;
  s.flag = reinterpret_cast<int*>(p);
  return s;
}

// Bytes of carve_attn(Q).
__host__ __device__ constexpr size_t attn_smem(int Q) {
  return sizeof(float) * ((size_t)Q * DK * 4 + (size_t)Q * APOS + 3 * MAXQ + (size_t)NWARP * Q * DK) + 16;
}

// Scores of one chunk of keys (K rows in the ring slot) for Q queries.
template <int QM>
__device__ __forceinline__ void chunk_scores(const AttnSmem& s, const Q1Regs& qr, const __half* kt, int npos, int Q) {
  if (QM == 1) attn_scores_q1(qr, kt, npos, s.sc);
  else attn_scores_multi(s.q, kt, npos, Q, s.sc);
}

template <int QM>
__device__ void self_attn_stage(const PlanDev& pd, const CallArgs& a, Ring& ring, const Ctx& cx, int layer, int c,
                                uint8_t* work) {
  AttnSmem s = carve_attn(work, pd.Qmax);
  const int S = pd.S, D = pd.D, H = pd.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int u = c; u < pd.R * H; u += pd.P) {
    const int b = u / H, h = u % H;
    const int off = cx.offs[b];
    for (int idx = threadIdx.x; idx < S * DK; idx += NTHR) {
      const int q = idx / DK, d = idx % DK;
      const __half* row = pd.qkv + (long long)(b * S + q) * 3 * D + h * DK + d;
      s.q[q * DK + d] = __half2float(__ldcg(row)) * 0.125f;
      s.knew[q * DK + d] = __half2float(__ldcg(row + D));
      s.vnew[q * DK + d] = __half2float(__ldcg(row + 2 * D));
    }
    if (threadIdx.x < S) {
      s.mrun[threadIdx.x] = -INFINITY;
      s.lrun[threadIdx.x] = 0.f;
    }
    AttnAcc<QM> acc;
#pragma unroll
    for (int q = 0; q < QM; ++q) acc.o[q][0] = acc.o[q][1] = 0.f;
    csync();
    Q1Regs qr;
    if (QM == 1) qr = q1_load(s.q);
    for (int j0 = 0; j0 < off; j0 += pd.apos) {
      const int npos = off - j0 < pd.apos ? off - j0 : pd.apos;
      const __half* kt = reinterpret_cast<const __half*>(ring.wait());
      chunk_scores<QM>(s, qr, kt, npos, S);
      ring.release();
      csync();
      attn_softmax(s.sc, npos, S, s.mrun, s.lrun, s.alpha, [](int, int) { return true; });
      csync();
      const __half* vt = reinterpret_cast<const __half*>(ring.wait());
      attn_accum<QM>(acc, s.sc, s.alpha, vt, npos, S);
      ring.release();
      csync();
    }
    // the new tokens, causally (keys/values from the QKV projection): a warp per (query, key) dot product
    for (int pr = warp; pr < S * S; pr += NWARP) {
      const int q = pr / S, j = pr % S;
      float sum = s.q[q * DK + lane] * s.knew[j * DK + lane] + s.q[q * DK + lane + 32] * s.knew[j * DK + lane + 32];
#pragma unroll
      for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (lane == 0) s.sc[q * APOS + j] = sum;
    }
    csync();
    attn_softmax(s.sc, S, S, s.mrun, s.lrun, s.alpha, [](int q, int j) { return j <= q; });
    csync();
#pragma unroll
    for (int q = 0; q < QM; ++q)
      if (q < S) {
        acc.o[q][0] *= s.alpha[q];
        acc.o[q][1] *= s.alpha[q];
      }
    for (int j = warp; j < S; j += NWARP) {
      const float2 v = make_float2(s.vnew[j * DK + 2 * lane], s.vnew[j * DK + 2 * lane + 1]);
#pragma unroll
      for (int q = 0; q < QM; ++q)
        if (q < S) {
          const float p = s.sc[q * APOS + j];
          acc.o[q][0] += p * v.x;
          acc.o[q][1] += p * v.y;
        }
    }
    attn_reduce<QM>(acc, S, s.scratch, s.out);
    // outputs: o (B-fragment order for the out-projection), the cache slots, new_kv
    for (int idx = threadIdx.x; idx < S * (DK / 2); idx += NTHR) {
      const int q = idx / (DK / 2), d = (idx % (DK / 2)) * 2;
      const float inv = 1.f / s.lrun[q];
      const int m = b * S + q;
      *reinterpret_cast<__half2*>(&pd.oB[bfrag_idx(m, h * DK + d, pd.NT)]) =
          __floats2half2_rn(s.out[q * DK + d] * inv, s.out[q * DK + d + 1] * inv);
      // (fp16 -> fp32 -> fp16 is exact: the cache gets the projection's fp16 values)
      const __half2 kn = __floats2half2_rn(s.knew[q * DK + d], s.knew[q * DK + d + 1]);
      const __half2 vn = __floats2half2_rn(s.vnew[q * DK + d], s.vnew[q * DK + d + 1]);
      const long long cslot = ((((long long)layer * pd.R + b) * H + h) * pd.C + off + q) * DK + d;
      *reinterpret_cast<__half2*>(a.kc + cslot) = kn;
      *reinterpret_cast<__half2*>(a.vc + cslot) = vn;
      const long long nk = ((((long long)layer * 2 * pd.R + b) * H + h) * S + q) * DK + d;
      const long long nv = nk + (long long)pd.R * H * S * DK;
      *reinterpret_cast<__half2*>(a.new_kv + nk) = kn;
      *reinterpret_cast<__half2*>(a.new_kv + nv) = vn;
    }
    csync();
  }
}

// Cross-attention: every CTA computes its pieces (frames of one (utterance, head) segment) and stores the
// partial softmax (unnormalised output, running max, running sum) per query in xpart[seg][rank]; the
// out-projection stage combines a segment's partials in rank order while it stages its B operand.
template <int QM>
__device__ void cross_attn_stage(const PlanDev& pd, const CallArgs& a, Ring& ring, int layer, int c, uint8_t* work,
                                 const Frames& fr) {
  AttnSmem s = carve_attn(work, pd.Qmax);
  const int S = pd.S, D = pd.D, H = pd.H, G = pd.G, Q = G * S;
  long long f0 = fr.bound(c), f1 = fr.bound(c + 1);
  Piece p;
  while (next_piece(fr, f0, f1, p)) {
    const int u = p.u, h = p.h;
    for (int idx = threadIdx.x; idx < Q * DK; idx += NTHR) {
      const int q = idx / DK, d = idx % DK;
      const int m = u * Q + q;  // rows u*G .. u*G+G-1, tokens s: token index (u*G + q/S)*S + q%S = u*Q + q
      s.q[q * DK + d] = __half2float(__ldcg(pd.q2 + (long long)m * D + h * DK + d)) * 0.125f;
    }
    if (threadIdx.x < Q) {
      s.mrun[threadIdx.x] = -INFINITY;
      s.lrun[threadIdx.x] = 0.f;
    }
    AttnAcc<QM> acc;
#pragma unroll
    for (int q = 0; q < QM; ++q) acc.o[q][0] = acc.o[q][1] = 0.f;
    csync();
    Q1Regs qr;
    if (QM == 1) qr = q1_load(s.q);
    for (int j0 = p.t0; j0 < p.t1; j0 += pd.apos) {
      const int npos = p.t1 - j0 < pd.apos ? p.t1 - j0 : pd.apos;
      const __half* kt = reinterpret_cast<const __half*>(ring.wait());
      chunk_scores<QM>(s, qr, kt, npos, Q);
      ring.release();
      csync();
      attn_softmax(s.sc, npos, Q, s.mrun, s.lrun, s.alpha, [](int, int) { return true; });
      csync();
      const __half* vt = reinterpret_cast<const __half*>(ring.wait());
      attn_accum<QM>(acc, s.sc, s.alpha, vt, npos, Q);
      ring.release();
      csync();
    }
    attn_reduce<QM>(acc, Q, s.scratch, s.out);
    const int seg = u * H + h;
    const int len = fr.pre[u + 1] - fr.pre[u];
    const long long sbeg = (long long)H * fr.pre[u] + (long long)h * len;
    const int rank = c - fr.owner(sbeg);
    float* part = pd.xpart + (((long long)seg * pd.P + rank) * Q) * XPS;
    for (int idx = threadIdx.x; idx < Q * XPS; idx += NTHR) {
      const int q = idx / XPS, d = idx % XPS;
      const float v = d < DK ? s.out[q * DK + d] : (d == DK ? s.mrun[q] : (d == DK + 1 ? s.lrun[q] : 0.f));
      __stcg(part + idx, v);
    }
    csync();
  }
}

// Exclusive prefix sum of v[0 .. n) in shared memory (n <= NTHR * 8), all consumer threads.
__device__ void block_exclusive_scan(int* v, int n, int* warp_tot) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int per = (n + NTHR - 1) / NTHR;
  const int lo = tid * per, hi = min(n, lo + per);
  int local = 0;
  for (int i = lo; i < hi; ++i) local += v[i];
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_tot[warp] = incl;
  csync();
  int base = 0;
  for (int w = 0; w < warp; ++w) base += warp_tot[w];
  int run = base + incl - local;
  for (int i = lo; i < hi; ++i) {
    const int x = v[i];
    v[i] = run;
    run += x;
  }
  csync();
}

// The out-projection's B operand from the cross-attention partials. Segment (utterance, head) s has nc(s)
// contributors, whose partials lie contiguously at xpart[s][0 .. nc) (Q x XPS floats each). The segments are
// staged into shared memory a round at a time (as many whole segments as fit, every thread issuing its
// loads back to back: one L2 round trip per round), then for every (segment, query, pair of dims) the
// contributors are combined in rank order (online max / rescale), normalised, and written in B-fragment
// order (padding tokens zero). A segment larger than the staging area is read from L2 directly.
__device__ void combine_cross_to_frag(const PlanDev& pd, const Frames& fr, __half* bbuf, float* stage, int cap,
                                      int* offs_s, const Ctx& cx) {
  const int H = pd.H, Q = pd.G * pd.S, NT = pd.NT, M = pd.M;
  const int nseg = pd.U * H, row = Q * XPS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* wtot = offs_s + nseg + 1;
  for (int sg = threadIdx.x; sg < nseg; sg += NTHR) {
    const int u = sg / H, h = sg % H;
    const int len = fr.pre[u + 1] - fr.pre[u];
    const long long sbeg = (long long)H * fr.pre[u] + (long long)h * len;
    offs_s[sg] = (fr.owner(sbeg + len - 1) - fr.owner(sbeg) + 1) * row;  // floats of the segment
  }
  if (threadIdx.x == 0) offs_s[nseg] = 0;
  csync();
  block_exclusive_scan(offs_s, nseg + 1, wtot);  // offs_s[s] = dense offset, offs_s[nseg] = total
  event(cx, 40);
  int s0 = 0;
  while (s0 < nseg) {
    // the round: segments s0 .. s1 - 1 whose dense data fits `cap` floats (at least one segment)
    int lo = s0 + 1, hi = nseg;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (offs_s[mid] - offs_s[s0] <= cap) lo = mid; else hi = mid - 1;
    }
    const int s1 = lo;
    const bool direct = offs_s[s0 + 1] - offs_s[s0] > cap;  // one oversize segment: straight from L2
    if (!direct) {
      // a warp per segment, 16-byte asynchronous copies (all in flight at once, one wait)
      for (int sg = s0 + warp; sg < s1; sg += NWARP) {
        const float* src = pd.xpart + (long long)sg * pd.P * row;
        float* dst = stage + (offs_s[sg] - offs_s[s0]);
        const int n4 = (offs_s[sg + 1] - offs_s[sg]) >> 2;
        for (int i = lane; i < n4; i += 32) cp_async16(dst + 4 * i, src + 4 * i);
      }
      cp_async_wait_all();
      csync();
      event(cx, 41);
    }
    if (!direct) {
      // pass 1, a thread per (segment, query): the contributors' weights exp(m_r - max) / sum_r' exp(m_r' - max)
      // l_r' written over their max slots
      for (int it = threadIdx.x; it < (s1 - s0) * Q; it += NTHR) {
        const int sg = s0 + it / Q, q = it % Q;
        const int nc = (offs_s[sg + 1] - offs_s[sg]) / row;
        float* base = stage + (offs_s[sg] - offs_s[s0]) + q * XPS;
        float mx = -INFINITY;
        for (int r = 0; r < nc; ++r) mx = fmaxf(mx, base[r * row + DK]);
        float den = 0.f;
        for (int r = 0; r < nc; ++r) {
          const float mr = base[r * row + DK];
          den += mr > -INFINITY ? expf(mr - mx) * base[r * row + DK + 1] : 0.f;
        }
        const float inv = den > 0.f ? 1.f / den : 0.f;
        for (int r = 0; r < nc; ++r) {
          const float mr = base[r * row + DK];
          base[r * row + DK] = mr > -INFINITY ? expf(mr - mx) * inv : 0.f;
        }
      }
      csync();
    }
    // pass 2, a thread per (segment, query, pair of dims): the weighted sum in rank order
    const int items = (s1 - s0) * Q * (DK / 2);
    for (int it = threadIdx.x; it < items; it += NTHR) {
      const int dp = it % (DK / 2), q = (it / (DK / 2)) % Q, sg = s0 + it / ((DK / 2) * Q);
      const int nc = (offs_s[sg + 1] - offs_s[sg]) / row;
      float n0 = 0.f, n1 = 0.f;
      if (!direct) {
        const float* pr = stage + (offs_s[sg] - offs_s[s0]) + q * XPS;
        for (int r = 0; r < nc; ++r, pr += row) {
          const float w = pr[DK];
          const float2 v = *reinterpret_cast<const float2*>(pr + 2 * dp);
          n0 += w * v.x;
          n1 += w * v.y;
        }
      } else {  // straight from L2: the online form over the contributors
        const float* base = pd.xpart + (long long)sg * pd.P * row;
        float mx = -INFINITY, den = 0.f;
        for (int r = 0; r < nc; ++r) {
          const float* pr = base + r * row + q * XPS;
          const float mr = __ldcg(pr + DK), lr = __ldcg(pr + DK + 1);
          if (mr > -INFINITY) {
            const float m1 = fmaxf(mx, mr);
            const float sc = mx > -INFINITY ? expf(mx - m1) : 0.f, w = expf(mr - m1);
            den = den * sc + w * lr;
            n0 = n0 * sc + w * __ldcg(pr + 2 * dp);
            n1 = n1 * sc + w * __ldcg(pr + 2 * dp + 1);
            mx = m1;
          }
        }
        const float inv = den > 0.f ? 1.f / den : 0.f;
        n0 *= inv;
        n1 *= inv;
      }
      const int u = sg / H, h = sg % H;
      const int m = u * Q + q;
      *reinterpret_cast<__half2*>(&bbuf[bfrag_idx(m, h * DK + 2 * dp, NT)]) = __floats2half2_rn(n0, n1);
    }
    csync();
    event(cx, 42);
    s0 = s1;
  }
  for (int m = M + warp; m < NT * 8; m += NWARP)  // padding tokens
    for (int k = lane * 2; k < pd.D; k += 64) *reinterpret_cast<uint32_t*>(&bbuf[bfrag_idx(m, k, NT)]) = 0u;
}

// ------------------------------------------------------------------------------------------------ other stages
__device__ void embed_stage(const PlanDev& pd, const CallArgs& a, const Ctx& cx, int c) {
  const long long total = (long long)pd.M * pd.D;
  const long long lo = total * c / pd.P, hi = total * (c + 1) / pd.P;
  for (long long i = lo + threadIdx.x; i < hi; i += NTHR) {
    int m = (int)(i / pd.D), n = (int)(i % pd.D);
    int r = m / pd.S, s = m % pd.S;
    long long t = a.tok[(long long)r * a.tok_stride + s];
    t = t < 0 ? 0 : (t >= pd.V ? pd.V - 1 : t);
    long long pos = (long long)cx.offs[r] + s;
    pos = pos >= pd.max_pos ? pd.max_pos - 1 : pos;
    pd.x[i] = __half2float(pd.emb[t * pd.D + n]) * pd.xscale + pd.pe[pos * pd.D + n];
  }
}

// After the output stage: per-CTA argmax partials -> global; the last CTA to arrive reduces them (all
// partials loaded into shared memory at once, then a warp per token).
__device__ void argmax_finish(const PlanDev& pd, const CallArgs& a, int c, OutState& os, int* flag, uint8_t* work) {
  for (int m = threadIdx.x; m < pd.M; m += NTHR) {
    __stcg(pd.amax + (long long)c * pd.M + m, os.amax[m]);
    __stcg(pd.aidx + (long long)c * pd.M + m, os.aidx[m]);
  }
  __threadfence();
  csync();
  if (threadIdx.x == 0) *flag = (atom_acq_rel_add(&pd.ctr[2], 1) == (uint32_t)(pd.P - 1));
  csync();
  if (!*flag) return;
  const int n = pd.P * pd.M;
  float* sv = reinterpret_cast<float*>(work);
  int* si = reinterpret_cast<int*>(sv + n);
#pragma unroll 4
  for (int i = threadIdx.x; i < n; i += NTHR) {
    sv[i] = __ldcg(pd.amax + i);
    si[i] = __ldcg(pd.aidx + i);
  }
  csync();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int m = warp; m < pd.M; m += NWARP) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int q = lane; q < pd.P; q += 32) {
      const float v = sv[q * pd.M + m];
      const int i = si[q * pd.M + m];
      if (v > best || (v == best && i < bi)) { best = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) {
      a.pred[m] = bi == 0x7fffffff ? 0 : bi;
      si[m] = bi == 0x7fffffff ? 0 : bi;  // (this CTA's copy of the argmax, for the accepted-draft count)
    }
  }
  if (a.res) {
    // drafted tokens accepted per row (_Verify.accept, runtime.py:1269-1278): positions up to the head's end s
    // count as accepted, then each drafted token that equals the argmax before it and is not <eos>
    csync();
    const int W = pd.S;
    for (int r = threadIdx.x; r < pd.R; r += NTHR) {
      const int64_t* row = a.inp + (long long)r * a.inp_stride;
      const long long s = row[W + 3] < 0 ? 0 : row[W + 3];
      int end = 0;
      while (end < W - 1 && ((si[r * W + end] == row[1 + end] && row[1 + end] != a.eos) || end < s)) ++end;
      a.res[2 * r] = end - s;
      a.res[2 * r + 1] = si[r * W + end];
    }
  }
  if (threadIdx.x == 0) atomicExch(&pd.ctr[2], 0u);
}

__device__ void beam_partials(const PlanDev& pd, int c, OutState& os) {
  for (int m = threadIdx.x; m < pd.M; m += NTHR) {
    __stcg(pd.lmax + (long long)c * pd.M + m, os.rmax[m]);
    __stcg(pd.lsum + (long long)c * pd.M + m, os.rsum[m]);
    for (int j = 0; j < KTOP; ++j) {
      __stcg(pd.topv + ((long long)c * pd.M + m) * KTOP + j, os.topv[m * KTOP + j]);
      __stcg(pd.topi + ((long long)c * pd.M + m) * KTOP + j, os.topi[m * KTOP + j]);
    }
  }
}

constexpr float LOG_ZERO = -1.0e10f;

// BeamSession._select step 1 for utterance u (one CTA). Each CTA of the output stage left, per row, its top-K
// logits as a sorted list (topv / topi), the row's max and sum of exp (lmax / lsum). The rows' lse come from the
// partials; a candidate's value is score + (logit - lse) (log_softmax), LOG_ZERO for every id of an inactive row
// (represented by its first K ids, the ones the order picks among equals). The best K of all lists are the best
// of their heads, K times: each warp takes lists round-robin (a lane holds the heads of up to SEL_LPL lists) and
// pops its best head K times (a warp argmax per round), then warp 0 merges the warps' K best the same way:
// top-`beam` by (value desc, flat index asc). The lists arrive in shared memory by bulk copies (one per CTA of
// the output stage and array); the stage's code stays short (it runs once per call, from a cold instruction
// cache).
// (Out of line: its registers would otherwise compete with the rest of the kernel's allocation.)
constexpr int SEL_LPL = 8;  // lists per lane: P x K + K <= NTHR x SEL_LPL
__device__ __noinline__ void select_stage(const PlanDev& pd, const CallArgs& a, const Ctx& cx, int c, uint8_t* work) {
  const int K = pd.beam, V = pd.V, P = pd.P, M = pd.M;
  const int B = pd.R / K;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* bar = reinterpret_cast<uint64_t*>(work);        // the lists' copies
  float* lmx = reinterpret_cast<float*>(work + 16);          // [KTOP] row max of the logits
  float* lse = lmx + KTOP;                                   // [KTOP] log of the row's sum of exp(logit - max)
  float* rsc = lse + KTOP;                                   // [KTOP] the rows' scores (before this step)
  int* ract = reinterpret_cast<int*>(rsc + KTOP);            // [KTOP] the rows' active flags
  float* wv = reinterpret_cast<float*>(ract + KTOP);         // [NWARP][KTOP] the warps' best
  int* wi = reinterpret_cast<int*>(wv + NWARP * KTOP);
  float* pm = reinterpret_cast<float*>(wi + NWARP * KTOP);   // [K][P] the CTAs' row max, then sum
  float* ps = pm + K * P;
  float* cvv = reinterpret_cast<float*>(work + ((16 + sizeof(float) * (4 * KTOP + 2 * NWARP * KTOP + 2 * (size_t)K * P) +
                                                 15) & ~(size_t)15));  // [P][K][KTOP] the CTAs' lists: values
  int* cvi = reinterpret_cast<int*>(cvv + (size_t)P * K * KTOP);                          // ... then ids
  const uint32_t run = (uint32_t)K * KTOP * 4;  // bytes of one CTA's lists of the utterance's rows
  const int nl = P * K + K;                     // lists: (CTA q, row k), then one per inactive row
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  uint32_t ph = 0;
  for (int u = c; u < B; u += P) {
    csync();  // (the barrier's initialisation; the previous utterance's reads of the staging areas)
    if (threadIdx.x == 0) mbar_arrive_expect_tx(bar, 2 * run * (uint32_t)P);
    csync();
    for (int i = threadIdx.x; i < 2 * P; i += NTHR) {  // copy i: CTA i / 2's lists, values (even) or ids (odd)
      const int q = i >> 1;
      const size_t at = ((size_t)q * M + (size_t)u * K) * KTOP;
      if (i & 1) bulk_g2s(cvi + (size_t)q * K * KTOP, pd.topi + at, run, bar, policy_evict_first());
      else bulk_g2s(cvv + (size_t)q * K * KTOP, pd.topv + at, run, bar, policy_evict_first());
    }
    if (threadIdx.x < K) {
      rsc[threadIdx.x] = a.score[u * K + threadIdx.x];
      ract[threadIdx.x] = a.active[u * K + threadIdx.x] != 0;
    }
#pragma unroll 4
    for (int i = threadIdx.x; i < K * P; i += NTHR) {
      const int k = i / P, q = i - k * P, r = u * K + k;
      pm[i] = __ldcg(pd.lmax + (long long)q * M + r);
      ps[i] = __ldcg(pd.lsum + (long long)q * M + r);
    }
    csync();
    for (int k = warp; k < K; k += NWARP) {
      float mx = -INFINITY;
      for (int q = lane; q < P; q += 32) mx = fmaxf(mx, pm[k * P + q]);
#pragma unroll
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float sm = 0.f;
      for (int q = lane; q < P; q += 32)
        if (pm[k * P + q] > -INFINITY) sm += ps[k * P + q] * expf(pm[k * P + q] - mx);
#pragma unroll
      for (int o = 16; o; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
      if (lane == 0) {
        lmx[k] = mx;
        lse[k] = logf(sm);
      }
    }
    if (!mbar_wait(bar, ph, pd.max_spin)) atomicExch(pd.err, E_ERR_TIMEOUT);
    ph ^= 1u;
    csync();
    event(cx, 74);
    // entry e of list l as a candidate (value, flat id); (-inf, INT_MAX) past its end
    auto entry = [&](int l, int e, float& v, int& id) {
      v = -INFINITY;
      id = 0x7fffffff;
      if (l < 0 || e >= K) return;
      if (l < P * K) {
        const int k = l % K;
        const float x = cvv[(size_t)l * KTOP + e];
        if (ract[k] && x > -INFINITY) {
          v = rsc[k] + ((x - lmx[k]) - lse[k]);  // log_softmax = (x - max) - log(sum)
          id = k * V + cvi[(size_t)l * KTOP + e];
        }
      } else {
        const int k = l - P * K;
        if (!ract[k]) {
          v = LOG_ZERO;
          id = k * V + e;
        }
      }
    };
    // this thread's lists: l = threadIdx.x + NTHR * j, and their heads
    int hl[SEL_LPL], he[SEL_LPL];
    float hv[SEL_LPL];
    int hid[SEL_LPL];
#pragma unroll
    for (int j = 0; j < SEL_LPL; ++j) {
      const int l = threadIdx.x + NTHR * j;
      hl[j] = l < nl ? l : -1;
      he[j] = 0;
      entry(hl[j], 0, hv[j], hid[j]);
    }
#pragma unroll 1
    for (int sel = 0; sel < K; ++sel) {
      float bv = -INFINITY;
      int bi = 0x7fffffff, bj = -1;
#pragma unroll
      for (int j = 0; j < SEL_LPL; ++j)
        if (beats(hv[j], hid[j], bv, bi)) bv = hv[j], bi = hid[j], bj = j;
      float wv0 = bv;
      int wi0 = bi;
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, wv0, o);
        const int oi = __shfl_xor_sync(0xffffffffu, wi0, o);
        if (beats(ov, oi, wv0, wi0)) wv0 = ov, wi0 = oi;
      }
      if (lane == 0) wv[warp * KTOP + sel] = wv0, wi[warp * KTOP + sel] = wi0;
      if (bj >= 0 && bi == wi0 && bi != 0x7fffffff) {  // (flat ids are unique: one lane pops its list)
#pragma unroll
        for (int j = 0; j < SEL_LPL; ++j)
          if (j == bj) {
            ++he[j];
            entry(hl[j], he[j], hv[j], hid[j]);
          }
      }
    }
    event(cx, 75);
    csync();
    if (warp == 0) {  // the warps' K best, each sorted: lane w < NWARP walks warp w's list
      int e = 0;
      float v = -INFINITY;
      int id = 0x7fffffff;
      if (lane < NWARP) v = wv[lane * KTOP], id = wi[lane * KTOP];
      float outv = -INFINITY;
      int outi = 0x7fffffff;
#pragma unroll 1
      for (int sel = 0; sel < K; ++sel) {
        float bv = v;
        int bi = id;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (beats(ov, oi, bv, bi)) bv = ov, bi = oi;
        }
        if (lane == sel) outv = bv, outi = bi;
        if (lane < NWARP && id == bi && bi != 0x7fffffff) {
          ++e;
          v = e < K ? wv[lane * KTOP + e] : -INFINITY;
          id = e < K ? wi[lane * KTOP + e] : 0x7fffffff;
        }
      }
      // (the old rows' scores were staged above, before the CTA barriers)
      const int fi = outi == 0x7fffffff ? 0 : outi;
      if (lane < K) {
        a.score[u * K + lane] = outv;
        a.parent[u * K + lane] = (long long)u * K + fi / V;
        a.token[u * K + lane] = fi % V;
      }
      if (a.shared) {
        // The caller's record of the slots each pair (i, j) of the utterance's rows holds in common (before this
        // step's write): row i takes its parent's slots from D[i][parent] on (the ones before are the same), and
        // afterwards two rows hold in common all of a parent's slots when they share it, else what their parents
        // held in common. (K x K <= 64 entries: lane l holds entries l and l + 32.)
        int32_t* Dm = a.shared + (size_t)u * K * K;
        const int pl = lane < K ? fi / V : 0;  // row lane's parent (index in the utterance)
        const int kk = K * K;
        const int e0 = lane < kk ? Dm[lane] : 0, e1 = lane + 32 < kk ? Dm[lane + 32] : 0;
        auto old_at = [&](int idx) {  // entry idx of the old matrix (every lane passes its own idx)
          const int x0 = __shfl_sync(0xffffffffu, e0, idx & 31), x1 = __shfl_sync(0xffffffffu, e1, idx & 31);
          return idx < 32 ? x0 : x1;
        };
        const int cs = old_at(lane < K ? lane * K + pl : 0);
        if (lane < K) pd.cstart[u * K + lane] = cs;
        int nv[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int idx = lane + 32 * h, i = idx < kk ? idx / K : 0, j = idx < kk ? idx % K : 0;
          const int pi = __shfl_sync(0xffffffffu, pl, i), pj = __shfl_sync(0xffffffffu, pl, j);
          const int o = old_at(pi * K + pj);
          nv[h] = pi == pj ? cx.offs[u * K + pi] + pd.S : o;
        }
        __syncwarp();  // (every lane's reads of the old matrix are done)
        if (lane < kk) Dm[lane] = nv[0];
        if (lane + 32 < kk) Dm[lane + 32] = nv[1];
      }
    }
    event(cx, 77);
  }
  csync();
  if (threadIdx.x == 0) mbar_inval(bar);  // (the next stage uses this memory for other data)
}

// Bytes of the select stage's shared memory.
__host__ __device__ constexpr size_t select_smem(int K, int P) {
  return ((16 + sizeof(float) * (4 * KTOP + 2 * NWARP * KTOP + 2 * (size_t)K * P) + 15) & ~(size_t)15) +
         2 * sizeof(float) * (size_t)P * K * KTOP;
}

// Cache reorder (BeamSession._select: buf.index_select(1, parent), runtime.py:1412-1413) in one stage, in place,
// by bulk copies: row r's slots 0 .. offset(parent) + S - 1 become its parent's, for the rows whose parent is
// another row (the slots past that are written by later calls before any call reads them). An item is (layer,
// head, block of PB positions); a run is a changed row's keys or values in it. Thread i < 2 x (changed rows) owns
// run i of every item: it copies the parent's run into its part of a shared-memory buffer and arrives on the
// buffer's barrier (expecting its bytes); once the barrier completes -- every run of the item has landed -- it
// copies its part into the row's slots. So an item's reads all land before any of its writes, and items are
// disjoint: the copy is in place. Two buffers: an item's loads overlap the previous item's stores (a thread
// reuses its part of a buffer after its own stores from there have read it). The stage's free shared memory --
// the ring, idle after the output stage, and the work area -- holds the buffers; PB is as large as they allow.
__device__ __noinline__ void reorder_stage(const PlanDev& pd, const CallArgs& a, const Ctx& cx, int c, uint8_t* work) {
  const int N = pd.R, H = pd.H, S = pd.S;
  uint8_t* area = work - (pd.off_work - pd.off_ring);
  const size_t avail = (size_t)(pd.off_work - pd.off_ring) + (size_t)pd.work_bytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(area);  // [2] one per buffer
  int* info = reinterpret_cast<int*>(area + 16);      // [4] changed rows, longest parent length, PB, first slot
  int* spar = info + 4;                               // [N] the row's parent, -1 where it keeps its slots
  int* chg = spar + N;                                // [N] the changed rows
  int* scs = chg + N;                                 // [N] the row's first slot to copy (with the record)
  const size_t hdr = (32 + (size_t)12 * N + 127) & ~(size_t)127;
  for (int r = threadIdx.x; r < N; r += NTHR) {
    const long long p = __ldcg(reinterpret_cast<const long long*>(a.parent) + r);
    spar[r] = (p == r || p < 0 || p >= N) ? -1 : (int)p;
    scs[r] = a.shared && spar[r] >= 0 ? min(max(__ldcg(pd.cstart + r), 0), cx.offs[spar[r]] + S) : 0;
  }
  csync();
  const size_t bufsz = ((avail - hdr) / 2) & ~(size_t)127;
  if (threadIdx.x == 0) {
    int nch = 0, maxlen = 0, mincs = 0x7fffffff;
    for (int r = 0; r < N; ++r)
      if (spar[r] >= 0) {
        chg[nch++] = r;
        const int lp = cx.offs[spar[r]] + S;
        maxlen = max(maxlen, lp);
        mincs = min(mincs, scs[r]);
      }
    info[0] = nch;
    info[1] = maxlen;
    info[2] = nch ? (int)min((size_t)max(maxlen - mincs, 1), bufsz / ((size_t)nch * 2 * DK * 2)) : 0;
    info[3] = nch ? mincs : 0;
    if (nch > 0) {
      mbar_init(&bar[0], 2 * nch);
      mbar_init(&bar[1], 2 * nch);
      fence_barrier_init();
    }
    event(cx, 78);
  }
  csync();
  const int nch = info[0], maxlen = info[1], PB = info[2], s0 = info[3];
  const int i = threadIdx.x;
  if (nch > 0 && PB > 0 && i < 2 * nch) {
    const int r = chg[i >> 1], par = spar[r], lp = cx.offs[par] + S;
    // the slots before cs are the same in the row and its parent (with the caller's record, else none)
    const int cs = scs[r];
    __half* cache = (i & 1) ? a.vc : a.kc;
    const uint64_t pol = policy_evict_first();
    const int nblk = (maxlen - s0 + PB - 1) / PB, nitems = pd.L * H * nblk;  // blocks of slots from s0 on
    const size_t part = (size_t)i * PB * DK * 2;  // this thread's part of a buffer
    uint8_t* const buf0 = area + hdr + part;
    uint8_t* const buf1 = area + hdr + bufsz + part;
    const long long rowh = (long long)pd.C * DK;  // halves of one (layer, row, head) cache row
    // item it: its run's bytes (0: nothing of this row in the block) and its source / destination offsets
    auto run_of = [&](int it, long long& src, long long& dst) -> uint32_t {
      const int lh = it / nblk, b0 = s0 + (it - lh * nblk) * PB, l = lh / H, h = lh - l * H;
      const int p0 = max(b0, cs), n = min(b0 + PB, lp) - p0;
      src = (((long long)l * N + par) * H + h) * rowh + (long long)p0 * DK;
      dst = (((long long)l * N + r) * H + h) * rowh + (long long)p0 * DK;
      return n > 0 ? (uint32_t)n * DK * 2 : 0u;
    };
    auto load = [&](int it, uint8_t* buf, uint64_t* b) {
      long long src, dst;
      const uint32_t bytes = run_of(it, src, dst);
      if (bytes) {
        mbar_arrive_expect_tx(b, bytes);
        bulk_g2s(buf, cache + src, bytes, b, pol);
      } else {
        mbar_arrive(b);
      }
    };
    uint32_t ph0 = 0u, ph1 = 0u;
    if (c < nitems) load(c, buf0, &bar[0]);
    int k = 0;
    for (int it = c; it < nitems; it += pd.P, ++k) {
      const bool odd = k & 1;
      const int nit = it + pd.P;
      if (nit < nitems) {
        bulk_wait_read_all();  // this thread's stores from the other buffer (the item before) have read it
        load(nit, odd ? buf0 : buf1, odd ? &bar[0] : &bar[1]);
      }
      if (!mbar_wait(odd ? &bar[1] : &bar[0], odd ? ph1 : ph0, pd.max_spin)) {
        atomicExch(pd.err, E_ERR_TIMEOUT);
        break;
      }
      if (odd) ph1 ^= 1u;
      else ph0 ^= 1u;
      long long src, dst;
      const uint32_t bytes = run_of(it, src, dst);
      if (bytes) {
        fence_proxy_async_cta();
        bulk_s2g(cache + dst, odd ? buf1 : buf0, bytes);
        bulk_commit();
      }
    }
    bulk_wait_all();
  }
  event(cx, 79);
  csync();
}

// ------------------------------------------------------------------------------------------------ kernel
__device__ OutState carve_out(uint8_t* p, int M, bool beam) {
  OutState os;
  float* f = reinterpret_cast<float*>(p);
  os.amax = f; f += M;
  os.aidx = reinterpret_cast<int*>(f); f += M;
  os.rmax = f; f += M;
  os.rsum = f; f += M;
  os.topv = f; f += M * KTOP;
  os.topi = reinterpret_cast<int*>(f); f += M * KTOP;
  os.wamax = f; f += NWARP * M;
  os.waidx = reinterpret_cast<int*>(f); f += NWARP * M;
  os.wrmax = os.wrsum = os.wtopv = os.wtile = nullptr;
  os.wtopi = nullptr;
  if (beam) {
    os.wrmax = f; f += NWARP * M;
    os.wrsum = f; f += NWARP * M;
    os.wtopv = f; f += NWARP * M * KTOP;
    os.wtopi = reinterpret_cast<int*>(f); f += NWARP * M * KTOP;
    os.wtile = f;
  }
  return os;
}

__host__ __device__ constexpr size_t out_smem(int M, bool beam) {
  return sizeof(float) * ((size_t)M * (4 + 2 * KTOP) + (size_t)NWARP * M * 2 +
                          (beam ? (size_t)NWARP * M * (2 + 2 * KTOP + 16) : 0));
}

// The plan and the call's pointers are __grid_constant__ parameters: read from the constant bank where used,
// not held in registers across the stage loop.
template <int NT>
__global__ void __launch_bounds__(BLOCK, 1)
    decoder_kernel(const __grid_constant__ PlanDev pd, const __grid_constant__ CallArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + MAXSLOT;
  int* pre = reinterpret_cast<int*>(smem + pd.off_pre);
  uint8_t* ringdata = smem + pd.off_ring;
  uint8_t* work = smem + pd.off_work;
  const int c = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_stages = 8 * pd.L + 2 + (a.beam_mode ? 2 : 0);

  int* so = reinterpret_cast<int*>(smem + pd.off_sched);
  int* sb = so + NGEMM + 1;
  int* offs = reinterpret_cast<int*>(smem + pd.off_rows);
  if (threadIdx.x == 0) {
    for (int s = 0; s < pd.nslot; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NWARP);
    }
    fence_barrier_init();
    pre[0] = 0;
    for (int u = 0; u < pd.U; ++u) pre[u + 1] = pre[u] + utt_len(pd, a, u);
    so[0] = 0;
    for (int gi = 0; gi < NGEMM; ++gi) so[gi + 1] = so[gi] + (pd.goff[gi][c + 1] - pd.goff[gi][c]);
  }
  for (int r = threadIdx.x; r < pd.R; r += BLOCK) offs[r] = row_off_global(pd, a, r);
  __syncthreads();
  for (int gi = 0; gi < NGEMM; ++gi) {
    const int base = pd.goff[gi][c];
    for (int i = threadIdx.x; i < so[gi + 1] - so[gi]; i += BLOCK) sb[so[gi] + i] = pd.gblk[gi][base + i];
  }
  __syncthreads();
  unsigned long long* evlog =
      pd.ts ? pd.ts + (size_t)n_stages * pd.P * 4 + (size_t)c * NEV : nullptr;
  int* nev = reinterpret_cast<int*>(smem + pd.off_pre) + 1033;
  if (threadIdx.x == 0) *nev = pd.ev_from > 0 ? NEV : 0;  // (recording starts at stage ev_from)
  const Ctx cx{so, sb, offs, evlog, nev, reinterpret_cast<float*>(smem + pd.off_pre) + 1040};
  Frames fr;
  fr.total = (long long)pd.H * pre[pd.U];
  fr.U = pd.U;
  fr.H = pd.H;
  fr.P = (int)(fr.total < pd.P ? fr.total : pd.P);
  fr.pre = pre;

  if (warp == NWARP) {  // producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      uint32_t i = 0;
      bool dead = false;
      for (int g = 0; g < n_stages && !dead; ++g) {
        for_chunks(pd, a, fr, cx, g, c, [&](const void* src, uint32_t bytes) {
          if (dead) return;
          const int s = i % pd.nslot;
          if (!mbar_wait(&empty[s], ((i / pd.nslot) & 1) ^ 1, pd.max_spin)) {
            dead = true;
            atomicExch(pd.err, E_ERR_TIMEOUT);
            return;
          }
          // at most `inflight` copies outstanding: the rest of the memory system stays responsive to the
          // consumers' small loads (their latency grows with the bytes queued ahead of them)
          if (i >= (uint32_t)pd.inflight) {
            const uint32_t j = i - pd.inflight;
            if (!mbar_wait(&full[j % pd.nslot], (j / pd.nslot) & 1, pd.max_spin)) {
              dead = true;
              atomicExch(pd.err, E_ERR_TIMEOUT);
              return;
            }
          }
          mbar_arrive_expect_tx(&full[s], bytes);
          bulk_g2s(ringdata + (size_t)s * pd.sstride, src, bytes, &full[s], pol);
          ++i;
        });
      }
      // Wait for the copies still in flight (the consumers may have stopped waiting for them): the CTA
      // must not exit while the copy engine writes its shared memory. Copies always complete, so this
      // uses the default limit, not the (testable) call limit.
      const uint32_t first = i > (uint32_t)pd.nslot ? i - pd.nslot : 0;
      for (uint32_t j = first; j < i; ++j) mbar_wait(&full[j % pd.nslot], (j / pd.nslot) & 1, DEFAULT_SPIN);
    }
    return;
  }

  Ring ring{full, empty, ringdata, pd.nslot, pd.sstride, 0, pd.max_spin, pd.err, false, 0ull, pd.ts != nullptr};
  OutState os = carve_out(smem + pd.off_out, pd.M, a.beam_mode != 0);
  for (int m = threadIdx.x; m < pd.M; m += NTHR) {
    os.amax[m] = -INFINITY;
    os.aidx[m] = 0x7fffffff;
    os.rmax[m] = -INFINITY;
    os.rsum[m] = 0.f;
    for (int j = 0; j < KTOP; ++j) {
      os.topv[m * KTOP + j] = -INFINITY;
      os.topi[m * KTOP + j] = 0x7fffffff;
    }
  }
  int* flag = reinterpret_cast<int*>(smem + pd.off_pre) + 1032;  // after pre[]
  bool dead = false;
  for (int g = 0; g < n_stages; ++g) {
    int layer;
    const Kind k = stage_kind(pd, g, layer);
    unsigned long long* ts = pd.ts ? pd.ts + ((size_t)g * pd.P + c) * 4 : nullptr;
    if (cx.ev && threadIdx.x == 0 && g == pd.ev_from && g > 0) *cx.nev = 0;
    if (ts && threadIdx.x == 0) ts[0] = globaltimer();
    switch (k) {
      case K_EMBED: embed_stage(pd, a, cx, c); break;
      case K_SATT:
        if (pd.S == 1) self_attn_stage<1>(pd, a, ring, cx, layer, c, work);
        else self_attn_stage<MAXQ>(pd, a, ring, cx, layer, c, work);
        break;
      case K_XATT:
        if (pd.G * pd.S == 1) cross_attn_stage<1>(pd, a, ring, layer, c, work, fr);
        else cross_attn_stage<MAXQ>(pd, a, ring, layer, c, work, fr);
        break;
      case K_SELECT: select_stage(pd, a, cx, c, work); break;
      case K_REORDER: reorder_stage(pd, a, cx, c, work); break;
      default: gemm_stage<NT>(pd, a, ring, cx, fr, k, layer, c, work, os); break;
    }
    if (k == K_OUT) {
      csync();
      if (a.beam_mode) beam_partials(pd, c, os);
      else if (a.pred) argmax_finish(pd, a, c, os, flag, work);
    }
    if (ts && threadIdx.x == 0) ts[1] = globaltimer();
    if (g < n_stages - 1) grid_sync(pd, (uint32_t)(g + 1) * pd.P, dead);
    if (ts && threadIdx.x == 0) {
      ts[2] = globaltimer();
      ts[3] = ring.waited;
    }
    ring.waited = 0;
  }
  // the last CTA out resets the barrier counter for the next call
  csync();
  if (threadIdx.x == 0) {
    if (atom_acq_rel_add(&pd.ctr[1], 1) == (uint32_t)(pd.P - 1)) {
      atomicExch(&pd.ctr[1], 0u);
      atomicExch(&pd.ctr[0], 0u);
    }
  }
}

// ------------------------------------------------------------------------------------------------ packing
// Weights [N, K] (fp32 or fp16, row-major) -> fragment order of rows [row0, row0 + N) of the destination;
// optional column scale (LayerNorm gamma). One thread per (row block, k block, lane).
__global__ void pack_kernel(const void* __restrict__ w, int dtype, int N, int K, const float* __restrict__ gamma,
                            uint4* __restrict__ out, int row0, int bstride) {
  const long long kbs = K >> 4;
  const long long total = (long long)((N + 15) >> 4) * kbs * 32;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int lane = (int)(i & 31);
    const long long kb = (i >> 5) % kbs;
    const long long rb = (i >> 5) / kbs;
    const int g = lane >> 2, t = lane & 3;
    uint32_t regs[4];
    for (int r = 0; r < 4; ++r) {
      const int row = (int)(rb * 16) + g + (r & 1) * 8;
      const int col = (int)(kb * 16) + 2 * t + (r >> 1) * 8;
      float v0 = 0.f, v1 = 0.f;
      if (row < N) {
        const long long o = (long long)row * K + col;
        if (dtype == OWSM_DEC_F32) {
          v0 = reinterpret_cast<const float*>(w)[o];
          v1 = reinterpret_cast<const float*>(w)[o + 1];
        } else {
          v0 = __half2float(reinterpret_cast<const __half*>(w)[o]);
          v1 = __half2float(reinterpret_cast<const __half*>(w)[o + 1]);
        }
        if (gamma) {
          v0 *= gamma[col];
          v1 *= gamma[col + 1];
        }
      }
      __half2 h = __floats2half2_rn(v0, v1);
      regs[r] = *reinterpret_cast<uint32_t*>(&h);
    }
    const long long dst = (long long)((row0 >> 4) + rb) * bstride + kb * 32 + lane;
    out[dst] = make_uint4(regs[0], regs[1], regs[2], regs[3]);
  }
}

// out[n] = b[n] + sum_k W[n, k] beta[k] (beta may be NULL): the bias after a folded LayerNorm. Warp per row.
__global__ void fold_bias_kernel(const void* __restrict__ w, int dtype, int N, int K, const float* __restrict__ beta,
                                 const float* __restrict__ b, float* __restrict__ out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= N) return;
  float s = 0.f;
  if (beta) {
    for (int k = lane; k < K; k += 32) {
      const long long o = (long long)warp * K + k;
      const float wv = dtype == OWSM_DEC_F32 ? reinterpret_cast<const float*>(w)[o]
                                             : __half2float(reinterpret_cast<const __half*>(w)[o]);
      s += wv * beta[k];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  }
  if (lane == 0) out[warp] = (b ? b[warp] : 0.f) + s;
}

__global__ void to_half_kernel(const void* __restrict__ src, int dtype, long long n, __half* __restrict__ dst) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    dst[i] = dtype == OWSM_DEC_F32 ? __float2half_rn(reinterpret_cast<const float*>(src)[i])
                                   : reinterpret_cast<const __half*>(src)[i];
}

// Folded biases [N] -> the 16-float tail of each 16-row block of the packed stream.
__global__ void place_bias_kernel(const float* __restrict__ b, int N, uint4* __restrict__ out, int bstride, int kbs) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float* tail = reinterpret_cast<float*>(out + (long long)(n >> 4) * bstride + (long long)kbs * 32);
  tail[n & 15] = b[n];
}

}  // namespace owsm

#include "cluster.cuh"
#include "dense.cuh"

// ================================================================================================ host / C ABI
using namespace owsm;

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

#define CUDA_TRY(x)                                                                              \
  do {                                                                                           \
    cudaError_t e_ = (x);                                                                        \
    if (e_ != cudaSuccess) return fail(OWSM_DEC_ERR_CUDA, std::string(#x ": ") + cudaGetErrorString(e_)); \
  } while (0)

struct DevBuf {
  void* p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
};

}  // namespace

namespace owsm {
// The library's last-error record for the other translation units (the K/V projection).
int record_error(int code, const std::string& msg) { return fail(code, msg); }
}  // namespace owsm

static std::atomic<uint64_t> g_handle_serial{0};

struct OwsmDec {
  uint64_t serial = ++g_handle_serial;  // tells handles apart even when one is freed and its address reused
  int device = 0;
  int programs = 0;
  int sms = 0;
  OwsmDecDims dims{};
  std::vector<void*> allocs;  // packed weights, biases, tables
  GemmW g[NGEMM]{};
  __half* emb = nullptr;
  float* pe = nullptr;
  int* err = nullptr;  // device error word
  uint32_t max_spin = DEFAULT_SPIN;
  int path = 0;  // 0: cluster kernel where it applies, 1: always the grid-stage kernel, 2: cluster kernel or fail,
                 // 3: dense kernel or fail
  __half* gt[NGEMM] = {};  // weights in 128-row tiles for the dense kernel (made by its first plan)
  long long gtl[NGEMM] = {};
  float* gcs[NGEMM] = {};  // their row sums, for the GEMMs after a LayerNorm
  // Profiling aid: with OWSM_DEC_NO_COOP set when the handle is made, cluster-kernel calls are launched
  // without the cooperative attribute (the profiler rejects cooperative cluster launches). The grid-wide
  // barrier then relies on all CTAs being resident, which holds when the call runs alone (one CTA per SM,
  // at most the resident cluster count); if they were not, its bounded waits report a timeout.
  bool coop = std::getenv("OWSM_DEC_NO_COOP") == nullptr;
  ~OwsmDec() {
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(device);
    for (void* p : allocs) cudaFree(p);
    cudaSetDevice(cur);
  }
};

struct OwsmDecPlan {
  OwsmDec* h = nullptr;
  PlanDev pd{};
  std::vector<void*> allocs;
  size_t smem = 0;
  int64_t scratch_bytes = 0;
  int beam = 0;
  // a call of more than 16 tokens on the cluster kernel: consecutive row slices of whole utterances, one
  // cluster-kernel launch each on the same stream (first row of each)
  std::vector<OwsmDecPlan*> subs;
  std::vector<int> sub_r0;
  size_t tcnt_bytes = 0;  // dense kernel: the per-tile arrival counters (reset after a failed call)
  ~OwsmDecPlan() {
    for (OwsmDecPlan* q : subs) delete q;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(h->device);
    for (void* p : allocs) cudaFree(p);
    cudaSetDevice(cur);
  }
};

namespace {

struct DeviceGuard {
  int prev = 0;
  explicit DeviceGuard(int d) {
    cudaGetDevice(&prev);
    cudaSetDevice(d);
  }
  ~DeviceGuard() { cudaSetDevice(prev); }
};

template <class T>
int dev_alloc(std::vector<void*>& list, T** out, size_t count, int64_t* total = nullptr) {
  void* p = nullptr;
  size_t bytes = count * sizeof(T);
  if (bytes == 0) bytes = 16;
  CUDA_TRY(cudaMalloc(&p, bytes));
  CUDA_TRY(cudaMemset(p, 0, bytes));
  list.push_back(p);
  *out = reinterpret_cast<T*>(p);
  if (total) *total += (int64_t)bytes;
  return OWSM_DEC_OK;
}

int launch_pack(const void* w, int dtype, int N, int K, const float* gamma, uint4* out, int row0, int bstride) {
  if (!w) return fail(OWSM_DEC_ERR_ARG, "missing weight pointer");
  long long total = (long long)((N + 15) / 16) * (K / 16) * 32;
  int blocks = (int)std::min<long long>((total + 255) / 256, 65535);
  pack_kernel<<<blocks, 256>>>(w, dtype, N, K, gamma, out, row0, bstride);
  CUDA_TRY(cudaGetLastError());
  return OWSM_DEC_OK;
}

int launch_fold(const void* w, int dtype, int N, int K, const float* beta, const float* b, float* out) {
  if (!w) return fail(OWSM_DEC_ERR_ARG, "missing weight pointer");
  int blocks = (N * 32 + 255) / 256;
  fold_bias_kernel<<<blocks, 256>>>(w, dtype, N, K, beta, b, out);
  CUDA_TRY(cudaGetLastError());
  return OWSM_DEC_OK;
}

}  // namespace

namespace {

// Greedy assignment of every 16-row block of the six layer GEMMs to the CTAs (largest blocks first, to the
// CTA with the fewest bytes so far): balanced bytes per CTA over a layer, which is what the streaming
// producers see. The output layer is split in contiguous ranges.
void assign_blocks(const GemmW* g, int P, std::vector<int> off[NGEMM], std::vector<int> blk[NGEMM]) {
  struct Item {
    long long bytes;
    int gi, rb;
  };
  std::vector<Item> items;
  for (int gi = 0; gi < G_OUT; ++gi)
    for (int rb = 0; rb < g[gi].NB; ++rb) items.push_back({(long long)g[gi].K * 32, gi, rb});
  std::stable_sort(items.begin(), items.end(), [](const Item& x, const Item& y) { return x.bytes > y.bytes; });
  std::vector<long long> load(P, 0);
  std::vector<std::vector<int>> per[NGEMM];
  for (int gi = 0; gi < NGEMM; ++gi) per[gi].assign(P, {});
  for (const Item& it : items) {
    int best = 0;
    for (int c = 1; c < P; ++c)
      if (load[c] < load[best]) best = c;
    load[best] += it.bytes;
    per[it.gi][best].push_back(it.rb);
  }
  for (int c = 0; c < P; ++c) {
    long long lo = (long long)g[G_OUT].NB * c / P, hi = (long long)g[G_OUT].NB * (c + 1) / P;
    for (long long rb = lo; rb < hi; ++rb) per[G_OUT][c].push_back((int)rb);
  }
  for (int gi = 0; gi < NGEMM; ++gi) {
    off[gi].assign(P + 1, 0);
    blk[gi].clear();
    for (int c = 0; c < P; ++c) {
      std::sort(per[gi][c].begin(), per[gi][c].end());
      off[gi][c + 1] = off[gi][c] + (int)per[gi][c].size();
      blk[gi].insert(blk[gi].end(), per[gi][c].begin(), per[gi][c].end());
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

using KernelFn = void (*)(PlanDev, CallArgs);

KernelFn kernel_for(int NT) {
  switch (NT) {
    case 1: return decoder_kernel<1>;
    case 2: return decoder_kernel<2>;
    case 4: return decoder_kernel<4>;
    default: return decoder_kernel<8>;
  }
}

// One instantiation per (token tiles, bound on the queries of an attention unit, beam): the per-query state
// of the attention code lives in registers, so a tighter bound leaves more registers to the rest.
KernelFn cl_kernel_for(int NT, int Qmax, bool beam, bool wide) {
  if (beam && wide) return NT == 1 ? decoder_cl_kernel<1, 1, true, true> : decoder_cl_kernel<2, 1, true, true>;
  if (beam) return NT == 1 ? decoder_cl_kernel<1, 1, true, false> : decoder_cl_kernel<2, 1, true, false>;
  if (Qmax == 1 && wide) return NT == 1 ? decoder_cl_kernel<1, 1, false, true> : decoder_cl_kernel<2, 1, false, true>;
  if (Qmax == 1) return NT == 1 ? decoder_cl_kernel<1, 1, false, false> : decoder_cl_kernel<2, 1, false, false>;
  if (Qmax <= 8) return NT == 1 ? decoder_cl_kernel<1, 8, false, false> : decoder_cl_kernel<2, 8, false, false>;
  return NT == 1 ? decoder_cl_kernel<1, CLQ, false, false> : decoder_cl_kernel<2, CLQ, false, false>;
}

KernelFn dense_kernel_for(int Qmax) {
  return Qmax == 1 ? decoder_dense_kernel<1, true> : decoder_dense_kernel<CLQ, false>;
}

KernelFn plan_kernel(const PlanDev& pd) {
  if (pd.dense) return dense_kernel_for(pd.Qmax);
  return pd.cl ? cl_kernel_for(pd.NT, pd.Qmax, pd.beam > 0, pd.wide != 0) : kernel_for(pd.NT);
}


}  // namespace

extern "C" {

const char* owsm_dec_last_error(void) { return g_last_error.c_str(); }

int owsm_dec_create(const OwsmDecDims* dims, const OwsmDecWeights* w, int device, int programs, OwsmDec** out) {
  if (!dims || !w || !out) return fail(OWSM_DEC_ERR_ARG, "null argument");
  *out = nullptr;
  const OwsmDecDims d = *dims;
  if (d.L < 1 || d.H < 1 || d.D != d.H * DK) return fail(OWSM_DEC_ERR_LIMIT, "the head size must be 64 (D = 64 * H)");
  if (d.D % 128 || d.D > 1024) return fail(OWSM_DEC_ERR_LIMIT, "d_model must be a multiple of 128, at most 1024");
  if (d.D % 16 || d.F % 16 || d.F < 16 || d.V < 1 || d.max_pos < 1)
    return fail(OWSM_DEC_ERR_LIMIT, "D and F must be multiples of 16");
  if (w->weight_dtype != OWSM_DEC_F32 && w->weight_dtype != OWSM_DEC_F16)
    return fail(OWSM_DEC_ERR_ARG, "weight_dtype must be OWSM_DEC_F32 or OWSM_DEC_F16");
  if (!w->layers || !w->emb || !w->pe || !w->wout) return fail(OWSM_DEC_ERR_ARG, "missing weights");
  DeviceGuard guard(device);
  cudaDeviceProp prop;
  CUDA_TRY(cudaGetDeviceProperties(&prop, device));
  if (prop.major < 10) return fail(OWSM_DEC_ERR_LIMIT, "libowsmdec needs an sm_100 GPU (B200)");
  OwsmDec* h = new OwsmDec();
  h->device = device;
  h->dims = d;
  h->sms = prop.multiProcessorCount;
  h->programs = (programs > 0 && programs < h->sms) ? programs : h->sms;
  const int dt = w->weight_dtype;
  const int D = d.D, F = d.F, L = d.L, V = d.V;
  struct Spec {
    int N, K, layers;
  } spec[NGEMM] = {{3 * D, D, L}, {D, D, L}, {D, D, L}, {D, D, L}, {F, D, L}, {D, F, L}, {V, D, 1}};
  int rc = OWSM_DEC_OK;
  auto bail = [&](int code) {
    delete h;
    return code;
  };
  for (int gi = 0; gi < NGEMM; ++gi) {
    GemmW& gw = h->g[gi];
    gw.N = spec[gi].N;
    gw.K = spec[gi].K;
    gw.NB = (gw.N + 15) / 16;
    gw.bstride = (gw.K / 16) * 32 + 4;
    gw.lstride = (long long)gw.NB * gw.bstride;
    uint4* wp;
    float* bp;
    if ((rc = dev_alloc(h->allocs, &wp, (size_t)gw.lstride * spec[gi].layers))) return bail(rc);
    if ((rc = dev_alloc(h->allocs, &bp, (size_t)gw.N * spec[gi].layers))) return bail(rc);
    gw.w = wp;
    gw.b = bp;
  }
  for (int l = 0; l < L; ++l) {
    const OwsmDecLayer& ly = w->layers[l];
    uint4* wq = const_cast<uint4*>(h->g[G_QKV].w) + (long long)l * h->g[G_QKV].lstride;
    float* bq = const_cast<float*>(h->g[G_QKV].b) + (long long)l * 3 * D;
    if (ly.wk) {
      const void* ws[3] = {ly.wq, ly.wk, ly.wv};
      const float* bs[3] = {ly.bq, ly.bk, ly.bv};
      for (int i = 0; i < 3; ++i) {
        if ((rc = launch_pack(ws[i], dt, D, D, ly.ln1_g, wq, i * D, h->g[G_QKV].bstride))) return bail(rc);
        if ((rc = launch_fold(ws[i], dt, D, D, ly.ln1_b, bs[i], bq + i * D))) return bail(rc);
      }
    } else {
      if ((rc = launch_pack(ly.wq, dt, 3 * D, D, ly.ln1_g, wq, 0, h->g[G_QKV].bstride))) return bail(rc);
      if ((rc = launch_fold(ly.wq, dt, 3 * D, D, ly.ln1_b, ly.bq, bq))) return bail(rc);
    }
    struct One {
      int gi;
      const void* w;
      const float* b;
      const float* g;
      const float* beta;
    } ones[5] = {{G_WO, ly.wo, ly.bo, nullptr, nullptr},
                 {G_CQ, ly.wcq, ly.bcq, ly.ln2_g, ly.ln2_b},
                 {G_WCO, ly.wco, ly.bco, nullptr, nullptr},
                 {G_F1, ly.w1, ly.b1, ly.ln3_g, ly.ln3_b},
                 {G_F2, ly.w2, ly.b2, nullptr, nullptr}};
    for (const One& o : ones) {
      GemmW& gw = h->g[o.gi];
      uint4* wp = const_cast<uint4*>(gw.w) + (long long)l * gw.lstride;
      float* bp = const_cast<float*>(gw.b) + (long long)l * gw.N;
      if ((rc = launch_pack(o.w, dt, gw.N, gw.K, o.g, wp, 0, gw.bstride))) return bail(rc);
      if ((rc = launch_fold(o.w, dt, gw.N, gw.K, o.beta, o.b, bp))) return bail(rc);
    }
  }
  {
    GemmW& gw = h->g[G_OUT];
    if ((rc = launch_pack(w->wout, dt, V, D, w->lnf_g, const_cast<uint4*>(gw.w), 0, gw.bstride))) return bail(rc);
    if ((rc = launch_fold(w->wout, dt, V, D, w->lnf_b, w->bout, const_cast<float*>(gw.b)))) return bail(rc);
  }
  for (int gi = 0; gi < NGEMM; ++gi) {  // biases into the packed streams
    const GemmW& gw = h->g[gi];
    for (int l = 0; l < spec[gi].layers; ++l) {
      place_bias_kernel<<<(gw.N + 255) / 256, 256>>>(gw.b + (long long)l * gw.N, gw.N,
                                                     const_cast<uint4*>(gw.w) + (long long)l * gw.lstride, gw.bstride,
                                                     gw.K / 16);
    }
  }
  if (cudaGetLastError() != cudaSuccess) return bail(fail(OWSM_DEC_ERR_CUDA, "bias placement failed"));
  if ((rc = dev_alloc(h->allocs, &h->emb, (size_t)V * D))) return bail(rc);
  to_half_kernel<<<1024, 256>>>(w->emb, dt, (long long)V * D, h->emb);
  if (cudaGetLastError() != cudaSuccess) return bail(fail(OWSM_DEC_ERR_CUDA, "embedding copy failed"));
  if ((rc = dev_alloc(h->allocs, &h->pe, (size_t)d.max_pos * D))) return bail(rc);
  if (cudaMemcpy(h->pe, w->pe, (size_t)d.max_pos * D * sizeof(float), cudaMemcpyDeviceToDevice) != cudaSuccess)
    return bail(fail(OWSM_DEC_ERR_CUDA, "positional table copy failed"));
  if ((rc = dev_alloc(h->allocs, &h->err, 4))) return bail(rc);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return bail(fail(OWSM_DEC_ERR_CUDA, std::string("packing: ") + cudaGetErrorString(e)));
  *out = h;
  return OWSM_DEC_OK;
}

void owsm_dec_destroy(OwsmDec* h) { delete h; }

}  // extern "C"

// The plan of a call shape; with allow_cl the cluster kernel where the shape allows it.
static int plan_impl(OwsmDec* h, int R, int S, int C, int T, int rows_per_utt, int beam, bool allow_cl,
                     OwsmDecPlan** out) {
  if (!h || !out) return fail(OWSM_DEC_ERR_ARG, "null argument");
  *out = nullptr;
  const OwsmDecDims& d = h->dims;
  const int G = rows_per_utt < 1 ? 1 : rows_per_utt;
  if (R < 1 || S < 1 || C < S || T < 1) return fail(OWSM_DEC_ERR_ARG, "bad call shape");
  if (R % G) return fail(OWSM_DEC_ERR_ARG, "rows must be a multiple of rows_per_utt");
  const int M = R * S;
  if (M > MAXNT * 8) return fail(OWSM_DEC_ERR_LIMIT, "at most 64 tokens (rows x window) per call");
  if (S > MAXQ || G * S > MAXQ) return fail(OWSM_DEC_ERR_LIMIT, "rows_per_utt x window must be <= 32");
  if (beam) {
    if ((long long)h->programs * beam + beam > (long long)NTHR * SEL_LPL)
      return fail(OWSM_DEC_ERR_LIMIT, "beam calls: too many programs for the select stage's lists");
    if (beam < 1 || beam > KTOP || S != 1 || R % beam || G != beam)
      return fail(OWSM_DEC_ERR_LIMIT, "beam calls: S = 1, beam <= 8, rows = batch x beam, rows_per_utt = beam");
  }
  if (C + S > d.max_pos + C) return fail(OWSM_DEC_ERR_ARG, "bad cache");
  const int U = R / G;
  if (U > 1024) return fail(OWSM_DEC_ERR_LIMIT, "at most 1024 utterances");
  DeviceGuard guard(h->device);
  OwsmDecPlan* p = new OwsmDecPlan();
  p->h = h;
  p->beam = beam;
  PlanDev& pd = p->pd;
  pd.L = d.L; pd.D = d.D; pd.H = d.H; pd.F = d.F; pd.V = d.V; pd.max_pos = d.max_pos;
  pd.eps = d.eps; pd.xscale = d.xscale;
  pd.R = R; pd.S = S; pd.M = M; pd.NT = M <= 8 ? 1 : M <= 16 ? 2 : M <= 32 ? 4 : 8; pd.C = C; pd.T = T; pd.G = G; pd.U = U; pd.beam = beam;
  pd.Rs = R; pd.Us = U;
  pd.P = h->programs;
  pd.max_spin = h->max_spin;
  pd.emb = h->emb;
  pd.pe = h->pe;
  for (int gi = 0; gi < NGEMM; ++gi) pd.g[gi] = h->g[gi];
  pd.err = h->err;
  pd.Qmax = std::max(S, G * S);
  auto bail = [&](int code) {
    delete p;
    return code;
  };
  cudaDeviceProp prop0;
  CUDA_TRY(cudaGetDeviceProperties(&prop0, h->device));
  // The cluster kernel: greedy calls of up to 16 tokens. Clusters of 4 CTAs, as many as fit one per SM;
  // row groups so that heads x row groups <= clusters; the FFN split over the largest count of clusters that
  // divides F / 64 and keeps a cluster's hidden fragments within the exchange buffer.
  if (allow_cl && (!beam || pd.Qmax > 1) && M <= 16 && pd.Qmax <= CLQ && d.D % 64 == 0 && d.F % 64 == 0) {
    KernelFn kf = cl_kernel_for(pd.NT, beam ? 1 : pd.Qmax, beam > 0, false);
    CUDA_TRY(cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)prop0.sharedMemPerBlockOptin));
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = CS;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cfg.blockDim = dim3(BLOCK);
    cfg.dynamicSmemBytes = prop0.sharedMemPerBlockOptin;
    cfg.gridDim = dim3(CS);
    int ncl = 0;
    CUDA_TRY(cudaOccupancyMaxActiveClusters(&ncl, (void*)kf, &cfg));
    ncl = std::min(ncl, h->programs / CS);
    int ncl3 = 0;
    for (int q = 1; q <= ncl; ++q)
      if ((d.F / 64) % q == 0 && (size_t)(d.F / q / 16) * pd.NT * 256 <= (size_t)XQ_FLOATS * 4) ncl3 = q;
    if (ncl >= d.H && ncl3 > 0) {
      pd.cl = 1;
      pd.P = ncl * CS;
      pd.RG = std::max(1, std::min(ncl / d.H, U));
      pd.NCL3 = ncl3;
      pd.F3 = d.F / ncl3;
      if (beam) {
        // a beam call's hypotheses attend as one-query groups of one row each (the one-query attention code,
        // lighter on registers than the kernel for units of several queries); the `beam` groups of an
        // utterance read its one copy of cross K/V (pd.Us copies in the caller's buffers, as before)
        pd.G = 1;
        pd.U = R;
        pd.kvg = beam;
        pd.Qmax = 1;
        pd.RG = std::max(1, std::min(ncl / d.H, R));
      }
      // one-query calls whose cross-attention units reach 256 frames: the kernel with wide attention steps
      const int ngm = (pd.U + pd.RG - 1) / pd.RG, parts = ngm >= CS ? 1 : CS / ngm;
      pd.wide = pd.Qmax == 1 && T / parts >= 256;
    }
  }
  if (allow_cl && h->path == 2 && !pd.cl) return bail(fail(OWSM_DEC_ERR_LIMIT, "the cluster kernel does not take this call"));
  int rc;
  int64_t* tot = &p->scratch_bytes;
  // schedule
  std::vector<int> off[NGEMM], blk[NGEMM];
  assign_blocks(pd.g, pd.P, off, blk);
  for (int gi = 0; gi < NGEMM; ++gi) {
    int *o, *b;
    if ((rc = dev_alloc(p->allocs, &o, off[gi].size(), tot))) return bail(rc);
    if ((rc = dev_alloc(p->allocs, &b, std::max<size_t>(blk[gi].size(), 1), tot))) return bail(rc);
    CUDA_TRY(cudaMemcpy(o, off[gi].data(), off[gi].size() * 4, cudaMemcpyHostToDevice));
    if (!blk[gi].empty()) CUDA_TRY(cudaMemcpy(b, blk[gi].data(), blk[gi].size() * 4, cudaMemcpyHostToDevice));
    pd.goff[gi] = o;
    pd.gblk[gi] = b;
  }
  // scratch
  const int NT = pd.NT, P = pd.P, D = d.D, F = d.F, Q = G * S;
  if ((rc = dev_alloc(p->allocs, &pd.x, (size_t)M * D, tot))) return bail(rc);
  if ((rc = dev_alloc(p->allocs, &pd.qkv, (size_t)M * 3 * D, tot))) return bail(rc);
  if ((rc = dev_alloc(p->allocs, &pd.q2, (size_t)M * D, tot))) return bail(rc);
  if ((rc = dev_alloc(p->allocs, &pd.oB, (size_t)NT * 8 * D, tot))) return bail(rc);
  if ((rc = dev_alloc(p->allocs, &pd.hB, (size_t)NT * 8 * F, tot))) return bail(rc);
  if (pd.cl) {
    for (int i = 0; i < 3; ++i)
      if ((rc = dev_alloc(p->allocs, &pd.xf[i], (size_t)M * D, tot))) return bail(rc);
    pd.xfix = pd.xf[(3 * d.L) % 3];
  } else if ((rc = dev_alloc(p->allocs, &pd.xpart, (size_t)U * d.H * P * Q * XPS, tot))) {
    return bail(rc);
  }
  if ((rc = dev_alloc(p->allocs, &pd.xcnt, (size_t)pd.U * d.H, tot))) return bail(rc);
  if ((rc = dev_alloc(p->allocs, &pd.amax, (size_t)P * M, tot))) return bail(rc);
  if ((rc = dev_alloc(p->allocs, &pd.aidx, (size_t)P * M, tot))) return bail(rc);
  if ((rc = dev_alloc(p->allocs, &pd.ctr, 8, tot))) return bail(rc);
  if (beam) {
    if ((rc = dev_alloc(p->allocs, &pd.lmax, (size_t)P * M, tot))) return bail(rc);
    if ((rc = dev_alloc(p->allocs, &pd.lsum, (size_t)P * M, tot))) return bail(rc);
    if ((rc = dev_alloc(p->allocs, &pd.topv, (size_t)P * M * KTOP, tot))) return bail(rc);
    if ((rc = dev_alloc(p->allocs, &pd.topi, (size_t)P * M * KTOP, tot))) return bail(rc);
    if ((rc = dev_alloc(p->allocs, &pd.cstart, (size_t)R, tot))) return bail(rc);
  }
  // shared memory: barriers | utterance prefix sums + flag | block lists | row offsets | output-stage state |
  // ring | work area
  size_t max_blocks = 0;
  for (int c = 0; c < pd.P; ++c) {
    size_t n = 0;
    for (int gi = 0; gi < NGEMM; ++gi) n += off[gi][c + 1] - off[gi][c];
    max_blocks = std::max(max_blocks, n);
  }
  size_t off_pre = 256;
  size_t off_sched = (off_pre + 4 * 1072 + 127) & ~(size_t)127;
  size_t off_rows = (off_sched + 4 * (NGEMM + 1 + max_blocks) + 127) & ~(size_t)127;
  size_t off_out = (off_rows + 4 * (size_t)R + 127) & ~(size_t)127;
  size_t off_ring = (off_out + out_smem(M, beam > 0) + 1023) & ~(size_t)1023;
  // GEMM stages: the B operand staged in shared memory (LayerNorm stages always; the others when the copy
  // fits stage_b) + per-chunk partial sums of blocks longer than one chunk
  const size_t cand_f = (size_t)NT * std::max(D, F) * 16, cand_d = (size_t)NT * D * 16;
  pd.stage_b = (int)(cand_f <= 128 * 1024 ? cand_f : (cand_d <= 128 * 1024 ? cand_d : 0));
  // the work area for a given ring slot size (chunks of slot / 512 k-blocks)
  auto work_for = [&](size_t slot_bytes) {
    size_t gemm_work = 0;
    for (int gi = 0; gi < NGEMM; ++gi) {
      const GemmW& gw = pd.g[gi];
      const int kbs = gw.K / 16;
      const bool lnk = (gi == G_QKV || gi == G_CQ || gi == G_F1 || gi == G_OUT);
      const size_t bb = (size_t)NT * kbs * 256;
      size_t need = lnk ? bb : (bb <= (size_t)pd.stage_b ? bb : 0);
      const int kpc = std::min(kbs, (int)(slot_bytes / 512));
      const int cpu = (kbs + kpc - 1) / kpc;
      if (cpu > 1) {
        size_t mb = 0;
        for (int c = 0; c < pd.P; ++c) mb = std::max(mb, (size_t)(off[gi][c + 1] - off[gi][c]));
        need += mb * cpu * NT * 512 + mb * 64;
      }
      gemm_work = std::max(gemm_work, need);
    }
    size_t w = std::max(gemm_work, attn_smem(pd.Qmax));
    // the cross-out stage: its B operand + the segment table (+ staging for the partials, below)
    w = std::max(w, (size_t)NT * D * 16 + 4 * (size_t)(U * d.H + 16) + 256);
    w = std::max(w, sizeof(float) * 2 * (size_t)pd.P * M);  // argmax partials of all CTAs
    if (beam) w = std::max(w, select_smem(beam, pd.P));
    return w;
  };
  cudaDeviceProp prop;
  CUDA_TRY(cudaGetDeviceProperties(&prop, h->device));
  const size_t limit = prop.sharedMemPerBlockOptin;
  auto slots_left = [&](size_t w, size_t sl) { return off_ring + w > limit ? (size_t)0 : (limit - off_ring - w) / (sl + 128); };
  // 32 KB slots while at least 4 fit (up to 6); else 16 KB slots while 4 fit; else the larger of the two
  // that leaves at least 2 slots
  size_t slot = SLOT, work = work_for(SLOT);
  if (pd.cl) {  // stage buffers of the cluster kernel; its output stage as the grid kernel's; 32 KB slots
    work = std::max(cl_work_bytes(NT, D, pd.Qmax), (size_t)NT * (D / 16) * 256 + 16);
    work = std::max(work, sizeof(float) * 2 * (size_t)pd.P * M);
    if (beam) work = std::max(work, select_smem(beam, pd.P));
    if (slots_left(work, SLOT) < 2) return bail(fail(OWSM_DEC_ERR_LIMIT, "shared memory too small for the cluster kernel"));
  } else if (slots_left(work, SLOT) < 4) {
    const size_t w16 = work_for(SLOT / 2);
    if (slots_left(w16, SLOT / 2) >= 4 || slots_left(work, SLOT) < 2) slot = SLOT / 2, work = w16;
  }
  if (slots_left(work, slot) < 2) return bail(fail(OWSM_DEC_ERR_LIMIT, "shared memory too small"));
  // staging for the cross-attention partials of the cross-out stage: 16 KB more when that leaves the ring as
  // it is (segments that do not fit are read from L2)
  if (!pd.cl) {
    const size_t wco = (size_t)NT * D * 16 + 4 * (size_t)(U * d.H + 16) + 256 + 16384;
    if (slots_left(std::max(work, wco), slot) >= std::min<size_t>(slots_left(work, slot), 4)) work = std::max(work, wco);
  }
  int nslot = (int)std::min<size_t>((limit - off_ring - work) / (slot + 128), slot == SLOT ? 6 : 8);
  pd.nslot = nslot;
  pd.slot = (int)slot;
  pd.apos = (int)(slot / (DK * 2));
  pd.off_pre = (int)off_pre;
  pd.off_sched = (int)off_sched;
  pd.off_rows = (int)off_rows;
  pd.inflight = std::min(nslot, (int)(65536 / slot));  // 64 KB of copies in flight per CTA
  pd.off_out = (int)off_out;
  pd.off_ring = (int)off_ring;
  pd.sstride = (int)slot + 128;
  pd.off_work = (int)(off_ring + (size_t)nslot * pd.sstride);
  pd.work_bytes = (int)work;
  p->smem = (size_t)pd.off_work + work;
  // the attribute is per function: set it to the device maximum once, so plans of other sizes coexist
  CUDA_TRY(cudaFuncSetAttribute(plan_kernel(pd), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)limit));
  int per_sm = 0;
  CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, plan_kernel(pd), BLOCK, p->smem));
  if (per_sm < 1) return bail(fail(OWSM_DEC_ERR_LIMIT, "the kernel does not fit an SM"));
  // the block-table uploads are pageable copies on the legacy stream, possibly still in flight; calls launch
  // on the caller's stream (maybe a non-blocking one, unordered against the legacy stream): finish them now
  CUDA_TRY(cudaDeviceSynchronize());
  *out = p;
  return OWSM_DEC_OK;
}

// The handle's weights in 128-row tiles (from its fragment packing, on the device), once per handle.
static int make_tiles(OwsmDec* h) {
  if (h->gt[0]) return OWSM_DEC_OK;
  for (int gi = 0; gi < NGEMM; ++gi) {
    const GemmW& gw = h->g[gi];
    const int layers = gi == G_OUT ? 1 : h->dims.L;
    const long long per = (long long)((gw.N + DN_TILE - 1) / DN_TILE) * DN_TILE * gw.K;
    __half* t = nullptr;
    int rc = dev_alloc(h->allocs, &t, (size_t)per * layers);
    if (rc) return rc;
    tile_pack_kernel<<<1024, 256>>>(gw.w, gw.N, gw.K, gw.bstride, gw.lstride, layers, t, per);
    CUDA_TRY(cudaGetLastError());
    h->gt[gi] = t;
    h->gtl[gi] = per;
    if (gi == G_QKV || gi == G_CQ || gi == G_F1 || gi == G_OUT) {
      float* cs = nullptr;
      if ((rc = dev_alloc(h->allocs, &cs, (size_t)gw.N * layers))) return rc;
      tile_rowsum_kernel<<<(gw.N * layers + 255) / 256, 256>>>(t, gw.N, gw.K, layers, per, cs);
      CUDA_TRY(cudaGetLastError());
      h->gcs[gi] = cs;
    }
  }
  CUDA_TRY(cudaDeviceSynchronize());
  return OWSM_DEC_OK;
}

// The plan of a greedy call of up to 64 tokens on the dense kernel.
static int plan_dense(OwsmDec* h, int R, int S, int C, int T, int G, OwsmDecPlan** out) {
  if (!h || !out) return fail(OWSM_DEC_ERR_ARG, "null argument");
  *out = nullptr;
  const OwsmDecDims& d = h->dims;
  if (R < 1 || S < 1 || C < S || T < 1 || G < 1 || R % G) return fail(OWSM_DEC_ERR_ARG, "bad call shape");
  const int M = R * S, U = R / G, Q = G * S;
  if (M > DN_TOK) return fail(OWSM_DEC_ERR_LIMIT, "the dense kernel takes at most 64 tokens per launch");
  if (Q > CLQ) return fail(OWSM_DEC_ERR_LIMIT, "the dense kernel takes at most 16 queries per utterance");
  if (U > 1024) return fail(OWSM_DEC_ERR_LIMIT, "at most 1024 utterances");
  DeviceGuard guard(h->device);
  int rc = make_tiles(h);
  if (rc) return rc;
  OwsmDecPlan* p = new OwsmDecPlan();
  p->h = h;
  auto bail = [&](int code) {
    delete p;
    return code;
  };
  PlanDev& pd = p->pd;
  pd.L = d.L; pd.D = d.D; pd.H = d.H; pd.F = d.F; pd.V = d.V; pd.max_pos = d.max_pos;
  pd.eps = d.eps; pd.xscale = d.xscale;
  pd.R = R; pd.S = S; pd.M = M; pd.NT = DN_MT; pd.C = C; pd.T = T; pd.G = G; pd.U = U; pd.beam = 0;
  pd.Rs = R; pd.Us = U;
  pd.P = h->programs;
  pd.max_spin = h->max_spin;
  pd.emb = h->emb;
  pd.pe = h->pe;
  pd.err = h->err;
  pd.Qmax = std::max(S, Q);
  pd.dense = 1;
  const int P = pd.P;
  int max_tiles_split = 0, max_tiles = 0;
  for (int gi = 0; gi < NGEMM; ++gi) {
    pd.g[gi] = h->g[gi];
    pd.gt[gi] = h->gt[gi];
    pd.gtl[gi] = h->gtl[gi];
    pd.gcs[gi] = h->gcs[gi];
    pd.nsplit[gi] = dn_splits(h->g[gi].K);
    const int nt = (h->g[gi].N + DN_TILE - 1) / DN_TILE;
    max_tiles = std::max(max_tiles, nt);
    if (pd.nsplit[gi] > 1) max_tiles_split = std::max(max_tiles_split, nt * pd.nsplit[gi]);
  }
  // work items (tile, K range): the six layer GEMMs on consecutive CTA ranges (a CTA's items of one layer are
  // in different stages, so its ring streams them back to back), the output layer over all CTAs
  std::vector<std::vector<int>> per[NGEMM];
  for (int gi = 0; gi < NGEMM; ++gi) per[gi].assign(P, {});
  int base = 0;
  for (int gi = 0; gi < NGEMM; ++gi) {
    const int n = ((h->g[gi].N + DN_TILE - 1) / DN_TILE) * pd.nsplit[gi];
    for (int j = 0; j < n; ++j) per[gi][(gi == G_OUT ? j : base + j) % P].push_back(j);
    if (gi != G_OUT) base = (base + n) % P;
  }
  int64_t* tot = &p->scratch_bytes;
  size_t max_items = 0;
  for (int gi = 0; gi < NGEMM; ++gi) {
    std::vector<int> off(P + 1, 0), blk;
    for (int c = 0; c < P; ++c) {
      off[c + 1] = off[c] + (int)per[gi][c].size();
      blk.insert(blk.end(), per[gi][c].begin(), per[gi][c].end());
    }
    int *o, *b;
    if ((rc = dev_alloc(p->allocs, &o, off.size(), tot))) return bail(rc);
    if ((rc = dev_alloc(p->allocs, &b, std::max<size_t>(blk.size(), 1), tot))) return bail(rc);
    CUDA_TRY(cudaMemcpy(o, off.data(), off.size() * 4, cudaMemcpyHostToDevice));
    if (!blk.empty()) CUDA_TRY(cudaMemcpy(b, blk.data(), blk.size() * 4, cudaMemcpyHostToDevice));
    pd.goff[gi] = o;
    pd.gblk[gi] = b;
  }
  for (int c = 0; c < P; ++c) {
    size_t n = 0;
    for (int gi = 0; gi < NGEMM; ++gi) n += per[gi][c].size();
    max_items = std::max(max_items, n);
  }
  const int D = d.D, F = d.F;
  if ((rc = dev_alloc(p->allocs, &pd.x, (size_t)M * D, tot))) return bail(rc);
  if ((rc = dev_alloc(p->allocs, &pd.qkv, (size_t)M * 3 * D, tot))) return bail(rc);
  if ((rc = dev_alloc(p->allocs, &pd.q2, (size_t)M * D, tot))) return bail(rc);
  if ((rc = dev_alloc(p->allocs, &pd.obuf, (size_t)D * DN_TOK, tot))) return bail(rc);
  if ((rc = dev_alloc(p->allocs, &pd.hbuf, (size_t)F * DN_TOK, tot))) return bail(rc);
  if ((rc = dev_alloc(p->allocs, &pd.xstat, (size_t)(D / DN_TILE) * DN_TOK * 2, tot))) return bail(rc);
  if ((rc = dev_alloc(p->allocs, &pd.xop, (size_t)2 * D * DN_TOK, tot))) return bail(rc);
  if ((rc = dev_alloc(p->allocs, &pd.part, (size_t)std::max(max_tiles_split, 1) * DN_TOK * DN_TILE, tot))) return bail(rc);
  if ((rc = dev_alloc(p->allocs, &pd.tcnt, (size_t)max_tiles, tot))) return bail(rc);
  p->tcnt_bytes = (size_t)max_tiles * sizeof(uint32_t);
  if ((rc = dev_alloc(p->allocs, &pd.xcnt, (size_t)pd.U * d.H, tot))) return bail(rc);
  if ((rc = dev_alloc(p->allocs, &pd.amax, (size_t)P * M, tot))) return bail(rc);
  if ((rc = dev_alloc(p->allocs, &pd.aidx, (size_t)P * M, tot))) return bail(rc);
  if ((rc = dev_alloc(p->allocs, &pd.ctr, 8, tot))) return bail(rc);
  // shared memory: barriers | utterance prefix sums + flags | work items | row offsets | argmax state | ring | work
  int maxkr = 0;  // the largest operand part (features x 2 for the high / low residual parts)
  for (int gi = 0; gi < NGEMM; ++gi) {
    const int kr = h->g[gi].K / pd.nsplit[gi], hilo = dn_hilo(gi);
    maxkr = std::max(maxkr, (kr / dn_parts(kr, hilo)) * (hilo ? 2 : 1));
  }
  const size_t off_pre = 256;
  const size_t off_sched = (off_pre + 4 * 1072 + 127) & ~(size_t)127;
  const size_t off_rows = (off_sched + 4 * (NGEMM + 1 + max_items) + 127) & ~(size_t)127;
  const size_t off_out = (off_rows + 4 * (size_t)R + 127) & ~(size_t)127;
  const size_t off_stat = (off_out + out_smem(M, false) + 127) & ~(size_t)127;
  const size_t off_ring = (off_stat + DN_TOK * 2 * sizeof(float) + 1023) & ~(size_t)1023;
  size_t work = (size_t)DN_TOK * maxkr * 2;
  work = std::max(work, ((attn_smem(pd.Qmax) + 15) & ~(size_t)15) + sizeof(float) * (size_t)pd.Qmax * XPS);
  work = std::max(work, sizeof(float) * 2 * (size_t)P * M);  // the argmax partials of all CTAs
  cudaDeviceProp prop;
  CUDA_TRY(cudaGetDeviceProperties(&prop, h->device));
  const size_t limit = prop.sharedMemPerBlockOptin;
  // ring slots of exactly 32 KB (no bias tails here), so the work area -- the token operand, swizzled in 1024-byte
  // groups -- starts 1024-byte aligned
  if (off_ring + work + 2 * SLOT > limit) return bail(fail(OWSM_DEC_ERR_LIMIT, "shared memory too small for the dense kernel"));
  const int nslot = (int)std::min<size_t>((limit - off_ring - work) / SLOT, 6);
  pd.nslot = nslot;
  pd.slot = SLOT;
  pd.apos = SLOT / (DK * 2);
  pd.off_pre = (int)off_pre;
  pd.off_sched = (int)off_sched;
  pd.off_rows = (int)off_rows;
  pd.inflight = nslot;  // every slot may be in flight: a work item streams 128 KB of weights
  pd.off_out = (int)off_out;
  pd.off_stat = (int)off_stat;
  pd.off_ring = (int)off_ring;
  pd.sstride = SLOT;
  pd.off_work = (int)(off_ring + (size_t)nslot * pd.sstride);
  pd.work_bytes = (int)work;
  p->smem = (size_t)pd.off_work + work;
  CUDA_TRY(cudaFuncSetAttribute(plan_kernel(pd), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)limit));
  int per_sm = 0;
  CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, plan_kernel(pd), BLOCK, p->smem));
  if (per_sm < 1) return bail(fail(OWSM_DEC_ERR_LIMIT, "the dense kernel does not fit an SM"));
  CUDA_TRY(cudaDeviceSynchronize());  // the table uploads, before calls on any stream
  *out = p;
  return OWSM_DEC_OK;
}

extern "C" {

int owsm_dec_plan(OwsmDec* h, int R, int S, int C, int T, int rows_per_utt, int beam, OwsmDecPlan** out) {
  if (!h || !out) return fail(OWSM_DEC_ERR_ARG, "null argument");
  const int G = rows_per_utt < 1 ? 1 : rows_per_utt;
  // greedy calls of more than 32 tokens (or any, with path 3): the dense kernel (tcgen05 GEMMs), one launch for
  // up to 64 tokens, consecutive row slices of whole utterances of up to 64 tokens each beyond
  if (((h->path == 0 && R * S > 32) || h->path == 3) && !beam && R >= 1 && S >= 1 && R % G == 0 && G * S <= CLQ) {
    int rc = OWSM_DEC_OK;
    if (R * S <= DN_TOK) {
      rc = plan_dense(h, R, S, C, T, G, out);
    } else {
      const int per = (DN_TOK / (S * G)) * G;  // rows per slice
      OwsmDecPlan* p = new OwsmDecPlan();
      p->h = h;
      for (int r0 = 0; r0 < R && rc == OWSM_DEC_OK; r0 += per) {
        OwsmDecPlan* q = nullptr;
        rc = plan_dense(h, std::min(per, R - r0), S, C, T, G, &q);
        if (rc == OWSM_DEC_OK) {
          q->pd.Rs = R;
          q->pd.Us = R / G;
          p->subs.push_back(q);
          p->sub_r0.push_back(r0);
          p->scratch_bytes += q->scratch_bytes;
        }
      }
      if (rc == OWSM_DEC_OK) {
        p->pd = p->subs[0]->pd;
        p->pd.R = R;
        p->pd.M = R * S;
        *out = p;
      } else {
        delete p;
      }
    }
    if (rc == OWSM_DEC_OK || h->path == 3) return rc;
  }
  // more than 16 tokens, greedy: row slices of whole utterances on the cluster kernel (each slice <= 16
  // tokens), launched one after another; the grid-stage kernel if that cannot be laid out
  if (h->path != 1 && !beam && R >= 1 && S >= 1 && R * S > 16 && R * S <= MAXNT * 8 && R % G == 0 && G * S <= 16) {
    const int per = (16 / (S * G)) * G;  // rows per slice
    OwsmDecPlan* p = new OwsmDecPlan();
    p->h = h;
    int rc = OWSM_DEC_OK;
    for (int r0 = 0; r0 < R && rc == OWSM_DEC_OK; r0 += per) {
      OwsmDecPlan* q = nullptr;
      rc = plan_impl(h, std::min(per, R - r0), S, C, T, G, 0, true, &q);
      if (rc == OWSM_DEC_OK && !q->pd.cl) rc = OWSM_DEC_ERR_LIMIT;
      if (rc == OWSM_DEC_OK) {
        q->pd.Rs = R;
        q->pd.Us = R / G;
        p->subs.push_back(q);
        p->sub_r0.push_back(r0);
        p->scratch_bytes += q->scratch_bytes;
      } else if (q) {
        delete q;
      }
    }
    if (rc == OWSM_DEC_OK) {
      p->pd = p->subs[0]->pd;  // (for the info calls: programs, ring slots, kernel)
      p->pd.R = R;
      p->pd.M = R * S;
      *out = p;
      return OWSM_DEC_OK;
    }
    delete p;
    if (h->path == 2) return rc;
  }
  const int rc = plan_impl(h, R, S, C, T, rows_per_utt, beam, h->path != 1, out);
  // a call the cluster kernel cannot lay out (shared memory, clusters) runs on the grid-stage kernel
  if (rc == OWSM_DEC_ERR_LIMIT && h->path == 0) return plan_impl(h, R, S, C, T, rows_per_utt, beam, false, out);
  return rc;
}

void owsm_dec_plan_destroy(OwsmDecPlan* p) { delete p; }

static int launch(OwsmDecPlan* p, void* stream, const CallArgs& a) {
  DeviceGuard guard(p->h->device);
  p->pd.max_spin = p->h->max_spin;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = CS;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.gridDim = dim3(p->pd.P);
  cfg.blockDim = dim3(BLOCK);
  cfg.dynamicSmemBytes = p->smem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cfg.attrs = p->pd.cl && !p->h->coop ? attr + 1 : attr;
  cfg.numAttrs = p->pd.cl ? (p->h->coop ? 2 : 1) : 1;
  CUDA_TRY(cudaLaunchKernelEx(&cfg, plan_kernel(p->pd), p->pd, a));
  return OWSM_DEC_OK;
}

static int check_common(OwsmDecPlan* p, const int64_t* tokens, const int64_t* offset, void* self_k, void* self_v,
                        const void* cross_k, const void* cross_v, float* logits, void* new_kv) {
  if (!p || !tokens || !offset || !self_k || !self_v || !cross_k || !cross_v || !logits || !new_kv)
    return fail(OWSM_DEC_ERR_ARG, "null buffer");
  if (!aligned16(self_k) || !aligned16(self_v) || !aligned16(cross_k) || !aligned16(cross_v))
    return fail(OWSM_DEC_ERR_ARG, "K/V buffers must be 16-byte aligned");
  return OWSM_DEC_OK;
}

// A greedy call, with (inp != NULL) a verify call's extras: the argmax under the timestamp rules (rules != 0) and
// the drafted tokens accepted (res != NULL). Row slices: the same buffers, offset to each slice's first row.
static int step_impl(OwsmDecPlan* p, void* stream, const int64_t* tokens, int64_t tok_stride, const int64_t* offset,
                     int64_t off_stride, void* self_k, void* self_v, const void* cross_k, const void* cross_v,
                     const int32_t* enc_len, float* logits, void* new_kv, int64_t* pred, const uint8_t* notime,
                     int first_time, int last_time, const int64_t* inp, int64_t inp_stride, int rules, int eos,
                     int64_t* res) {
  if (!p->subs.empty()) {
    const PlanDev& d0 = p->subs[0]->pd;
    const long long H = d0.H, C = d0.C, T = d0.T, S = d0.S, V = d0.V, G = d0.G;
    for (size_t i = 0; i < p->subs.size(); ++i) {
      const long long r0 = p->sub_r0[i], u0 = r0 / G;
      const int rc = step_impl(
          p->subs[i], stream, tokens + r0 * tok_stride, tok_stride, offset + r0 * off_stride, off_stride,
          reinterpret_cast<__half*>(self_k) + r0 * H * C * DK, reinterpret_cast<__half*>(self_v) + r0 * H * C * DK,
          reinterpret_cast<const __half*>(cross_k) + u0 * H * T * DK,
          reinterpret_cast<const __half*>(cross_v) + u0 * H * T * DK, enc_len ? enc_len + u0 : nullptr,
          logits + r0 * S * V, reinterpret_cast<__half*>(new_kv) + r0 * H * S * DK, pred ? pred + r0 * S : nullptr,
          notime ? notime + r0 : nullptr, first_time, last_time, inp ? inp + r0 * inp_stride : nullptr, inp_stride,
          rules, eos, res ? res + 2 * r0 : nullptr);
      if (rc) return rc;
    }
    return OWSM_DEC_OK;
  }
  CallArgs a{};
  a.tok = tokens; a.tok_stride = tok_stride;
  a.off = offset; a.off_stride = off_stride;
  a.kc = reinterpret_cast<__half*>(self_k); a.vc = reinterpret_cast<__half*>(self_v);
  a.ck = reinterpret_cast<const __half*>(cross_k); a.cv = reinterpret_cast<const __half*>(cross_v);
  a.enc_len = enc_len;
  a.logits = logits; a.new_kv = reinterpret_cast<__half*>(new_kv);
  a.pred = pred; a.notime = notime; a.ft = first_time; a.lt = last_time;
  a.inp = inp; a.inp_stride = inp_stride; a.rules = rules; a.eos = eos; a.res = res;
  a.beam_mode = 0;
  return launch(p, stream, a);
}

int owsm_dec_step(OwsmDecPlan* p, void* stream, const int64_t* tokens, int64_t tok_stride, const int64_t* offset,
                  int64_t off_stride, void* self_k, void* self_v, const void* cross_k, const void* cross_v,
                  const int32_t* enc_len, float* logits, void* new_kv, int64_t* pred, const uint8_t* notime,
                  int first_time, int last_time) {
  const int rc = check_common(p, tokens, offset, self_k, self_v, cross_k, cross_v, logits, new_kv);
  if (rc) return rc;
  return step_impl(p, stream, tokens, tok_stride, offset, off_stride, self_k, self_v, cross_k, cross_v, enc_len,
                   logits, new_kv, pred, notime, first_time, last_time, nullptr, 0, 0, -1, nullptr);
}

int owsm_dec_step_verify(OwsmDecPlan* p, void* stream, const int64_t* inp, int64_t inp_stride, void* self_k,
                         void* self_v, const void* cross_k, const void* cross_v, const int32_t* enc_len,
                         float* logits, void* new_kv, int64_t* pred, const uint8_t* notime, int rules,
                         int first_time, int last_time, int eos, int64_t* res) {
  if (!p || !inp || !pred) return fail(OWSM_DEC_ERR_ARG, "owsm_dec_step_verify needs the input rows and pred");
  if (p->beam) return fail(OWSM_DEC_ERR_ARG, "a verify call needs a greedy plan");
  const int S = p->subs.empty() ? p->pd.S : p->subs[0]->pd.S;
  if (inp_stride < S + 4) return fail(OWSM_DEC_ERR_ARG, "input rows are [S tokens, offset, count, last, first]");
  if (rules && first_time > last_time) return fail(OWSM_DEC_ERR_ARG, "timestamp ids: first > last");
  const int rc = check_common(p, inp, inp + S, self_k, self_v, cross_k, cross_v, logits, new_kv);
  if (rc) return rc;
  return step_impl(p, stream, inp, inp_stride, inp + S, inp_stride, self_k, self_v, cross_k, cross_v, enc_len, logits,
                   new_kv, pred, notime, first_time, last_time, inp, inp_stride, rules ? 1 : 0, eos, res);
}

int owsm_dec_beam_step(OwsmDecPlan* p, void* stream, const int64_t* tokens, int64_t tok_stride,
                       const int64_t* offset, int64_t off_stride, void* self_k, void* self_v, const void* cross_k,
                       const void* cross_v, const int32_t* enc_len, float* logits, void* new_kv, float* score,
                       const uint8_t* active, int64_t* parent, int64_t* token, int32_t* shared) {
  int rc = check_common(p, tokens, offset, self_k, self_v, cross_k, cross_v, logits, new_kv);
  if (rc) return rc;
  if (!p->beam) return fail(OWSM_DEC_ERR_ARG, "the plan was not made for beam calls");
  if (!score || !active || !parent || !token) return fail(OWSM_DEC_ERR_ARG, "null beam buffer");
  CallArgs a{};
  a.tok = tokens; a.tok_stride = tok_stride;
  a.off = offset; a.off_stride = off_stride;
  a.kc = reinterpret_cast<__half*>(self_k); a.vc = reinterpret_cast<__half*>(self_v);
  a.ck = reinterpret_cast<const __half*>(cross_k); a.cv = reinterpret_cast<const __half*>(cross_v);
  a.enc_len = enc_len;
  a.logits = logits; a.new_kv = reinterpret_cast<__half*>(new_kv);
  a.score = score; a.active = active; a.parent = parent; a.token = token;
  a.shared = shared;
  a.beam_mode = 1;
  return launch(p, stream, a);
}

int owsm_dec_get_error(OwsmDec* h) {
  if (!h) return fail(OWSM_DEC_ERR_ARG, "null handle");
  DeviceGuard guard(h->device);
  CUDA_TRY(cudaDeviceSynchronize());
  int e = 0;
  CUDA_TRY(cudaMemcpy(&e, h->err, 4, cudaMemcpyDeviceToHost));
  if (e) {
    CUDA_TRY(cudaMemset(h->err, 0, 4));
    return fail(OWSM_DEC_ERR_TIMEOUT, "a bounded in-kernel wait gave up");
  }
  return OWSM_DEC_OK;
}

int owsm_dec_plan_reset(OwsmDecPlan* p) {
  if (!p) return fail(OWSM_DEC_ERR_ARG, "null plan");
  for (OwsmDecPlan* q : p->subs) {
    const int rc = owsm_dec_plan_reset(q);
    if (rc) return rc;
  }
  if (!p->subs.empty()) return OWSM_DEC_OK;
  DeviceGuard guard(p->h->device);
  CUDA_TRY(cudaDeviceSynchronize());
  CUDA_TRY(cudaMemset(p->pd.ctr, 0, 8 * sizeof(uint32_t)));
  CUDA_TRY(cudaMemset(p->pd.xcnt, 0, (size_t)p->pd.U * p->pd.H * sizeof(uint32_t)));
  if (p->tcnt_bytes) CUDA_TRY(cudaMemset(p->pd.tcnt, 0, p->tcnt_bytes));
  return OWSM_DEC_OK;
}

int owsm_dec_plan_info(const OwsmDecPlan* p, int* programs, int* ring_slots, int64_t* scratch_bytes) {
  if (!p) return fail(OWSM_DEC_ERR_ARG, "null plan");
  if (programs) *programs = p->pd.P;
  if (ring_slots) *ring_slots = p->pd.nslot;
  if (scratch_bytes) *scratch_bytes = p->scratch_bytes;
  return OWSM_DEC_OK;
}

int owsm_dec_plan_trace(OwsmDecPlan* p, void* stamps) {
  if (!p) return fail(OWSM_DEC_ERR_ARG, "null plan");
  if (!p->subs.empty()) return owsm_dec_plan_trace(p->subs[0], stamps);  // a sliced call: its first slice
  DeviceGuard guard(p->h->device);
  p->pd.ts = reinterpret_cast<unsigned long long*>(stamps);
  return OWSM_DEC_OK;
}

int owsm_dec_plan_trace_from(OwsmDecPlan* p, int first_stage) {
  if (!p || first_stage < 0) return fail(OWSM_DEC_ERR_ARG, "null plan or negative stage");
  if (!p->subs.empty()) return owsm_dec_plan_trace_from(p->subs[0], first_stage);
  p->pd.ev_from = first_stage;
  return OWSM_DEC_OK;
}

int owsm_dec_plan_stages(const OwsmDecPlan* p, int beam_call) {
  if (!p) return fail(OWSM_DEC_ERR_ARG, "null plan");
  return (p->pd.cl ? 3 * p->pd.L + 2 : 8 * p->pd.L + 2) + (beam_call ? 2 : 0);
}

int owsm_dec_set_path(OwsmDec* h, int path) {
  if (!h) return fail(OWSM_DEC_ERR_ARG, "null handle");
  if (path < 0 || path > 3) return fail(OWSM_DEC_ERR_ARG, "path must be 0, 1, 2 or 3");
  h->path = path;
  return OWSM_DEC_OK;
}

int owsm_dec_plan_kernel(const OwsmDecPlan* p) {
  if (!p) return fail(OWSM_DEC_ERR_ARG, "null plan");
  return p->pd.dense ? 3 : (p->pd.cl ? 2 : 1);
}

int owsm_dec_plan_launches(const OwsmDecPlan* p) {
  if (!p) return fail(OWSM_DEC_ERR_ARG, "null plan");
  return p->subs.empty() ? 1 : (int)p->subs.size();
}

int owsm_dec_set_max_spin(OwsmDec* h, uint32_t polls) {
  if (!h) return fail(OWSM_DEC_ERR_ARG, "null handle");
  h->max_spin = polls ? polls : DEFAULT_SPIN;
  return OWSM_DEC_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------ fixed scratch
// owsm_dec_step_static: the greedy call of owsm_dec_step for callers that must not allocate device memory
// when they decide to decode -- an audio or serving thread that may not block on cudaMalloc (it can
// synchronise the device and stall every stream of the process), or code whose device memory is owned by an
// outside pool that forbids allocations of its own. Its per-call scratch (residual stream, activations,
// cross-attention partials, argmax partials, barrier counters, block tables) lives in one array of this
// library per device, sized at compile time; nothing is allocated, not at set-up and not per call.
namespace {

constexpr size_t STATIC_SCRATCH_BYTES = (size_t)8 << 20;  // 8 MiB per device
constexpr int STATIC_MAX_TOKENS = 8;                       // rows x window per fixed-scratch call
constexpr int STATIC_MAX_DEVICES = 64;

// What one device's fixed scratch is laid out for: the handle and call shape of the last set-up.
struct StaticLayout {
  uint64_t serial = 0;  // handle serial (0: never set up)
  int R = 0, S = 0, C = 0, T = 0;
  uint8_t* base = nullptr;  // device address of owsm_static_scratch on this device
  PlanDev pd{};
  size_t smem = 0;
};
StaticLayout g_static[STATIC_MAX_DEVICES];
std::mutex g_static_mu;

}  // namespace

static __device__ __align__(256) uint8_t owsm_static_scratch[STATIC_SCRATCH_BYTES];

// The launch description of a greedy call of shape (R rows, S tokens, C cache slots, T frames, one row per
// utterance) with its scratch carved from `base`, as owsm_dec_plan builds it from allocations. Returns the
// bytes the carve needs in `need`; writes nothing to the device when `base` is null (a dry run) and uploads
// the block tables otherwise.
static int static_layout(OwsmDec* h, int R, int S, int C, int T, uint8_t* base, PlanDev& pd, size_t& smem,
                         size_t& need) {
  const OwsmDecDims& d = h->dims;
  const int M = R * S, U = R, Q = S;
  pd = PlanDev{};
  pd.L = d.L; pd.D = d.D; pd.H = d.H; pd.F = d.F; pd.V = d.V; pd.max_pos = d.max_pos;
  pd.eps = d.eps; pd.xscale = d.xscale;
  pd.R = R; pd.S = S; pd.M = M; pd.NT = M <= 8 ? 1 : 2; pd.C = C; pd.T = T; pd.G = 1; pd.U = U; pd.beam = 0;
  pd.P = h->programs;
  pd.max_spin = h->max_spin;
  pd.emb = h->emb;
  pd.pe = h->pe;
  for (int gi = 0; gi < NGEMM; ++gi) pd.g[gi] = h->g[gi];
  pd.err = h->err;
  pd.Qmax = S;
  const int NT = pd.NT, P = pd.P, D = d.D, F = d.F;
  std::vector<int> off[NGEMM], blk[NGEMM];  // host-side schedule (host memory only)
  assign_blocks(pd.g, P, off, blk);
  size_t at = 0;
  auto take = [&](size_t bytes) {
    at = (at + 255) & ~(size_t)255;
    uint8_t* q = base ? base + at : nullptr;
    at += bytes ? bytes : 16;
    return q;
  };
  for (int gi = 0; gi < NGEMM; ++gi) {
    pd.goff[gi] = reinterpret_cast<const int*>(take(off[gi].size() * 4));
    pd.gblk[gi] = reinterpret_cast<const int*>(take(std::max<size_t>(blk[gi].size(), 1) * 4));
  }
  pd.x = reinterpret_cast<float*>(take((size_t)M * D * 4));
  pd.qkv = reinterpret_cast<__half*>(take((size_t)M * 3 * D * 2));
  pd.q2 = reinterpret_cast<__half*>(take((size_t)M * D * 2));
  pd.oB = reinterpret_cast<__half*>(take((size_t)NT * 8 * D * 2));
  pd.hB = reinterpret_cast<__half*>(take((size_t)NT * 8 * F * 2));
  pd.xpart = reinterpret_cast<float*>(take((size_t)U * d.H * P * Q * XPS * 4));
  pd.xcnt = reinterpret_cast<uint32_t*>(take((size_t)U * d.H * 4));
  pd.amax = reinterpret_cast<float*>(take((size_t)P * M * 4));
  pd.aidx = reinterpret_cast<int*>(take((size_t)P * M * 4));
  pd.ctr = reinterpret_cast<uint32_t*>(take(8 * 4));
  need = at;
  if (need > STATIC_SCRATCH_BYTES) return OWSM_DEC_OK;  // the caller rejects the shape
  // shared memory, as owsm_dec_plan lays it out for a greedy call
  size_t max_blocks = 0;
  for (int c = 0; c < P; ++c) {
    size_t n = 0;
    for (int gi = 0; gi < NGEMM; ++gi) n += off[gi][c + 1] - off[gi][c];
    max_blocks = std::max(max_blocks, n);
  }
  const size_t off_pre = 256;
  const size_t off_sched = (off_pre + 4 * 1072 + 127) & ~(size_t)127;
  const size_t off_rows = (off_sched + 4 * (NGEMM + 1 + max_blocks) + 127) & ~(size_t)127;
  const size_t off_out = (off_rows + 4 * (size_t)R + 127) & ~(size_t)127;
  const size_t off_ring = (off_out + out_smem(M, false) + 1023) & ~(size_t)1023;
  const size_t cand_f = (size_t)NT * std::max(D, F) * 16, cand_d = (size_t)NT * D * 16;
  pd.stage_b = (int)(cand_f <= 128 * 1024 ? cand_f : (cand_d <= 128 * 1024 ? cand_d : 0));
  auto work_for = [&](size_t slot_bytes) {
    size_t gemm_work = 0;
    for (int gi = 0; gi < NGEMM; ++gi) {
      const GemmW& gw = pd.g[gi];
      const int kbs = gw.K / 16;
      const bool lnk = (gi == G_QKV || gi == G_CQ || gi == G_F1 || gi == G_OUT);
      const size_t bb = (size_t)NT * kbs * 256;
      size_t nd = lnk ? bb : (bb <= (size_t)pd.stage_b ? bb : 0);
      const int kpc = std::min(kbs, (int)(slot_bytes / 512));
      const int cpu = (kbs + kpc - 1) / kpc;
      if (cpu > 1) {
        size_t mb = 0;
        for (int c = 0; c < P; ++c) mb = std::max(mb, (size_t)(off[gi][c + 1] - off[gi][c]));
        nd += mb * cpu * NT * 512 + mb * 64;
      }
      gemm_work = std::max(gemm_work, nd);
    }
    size_t w = std::max(gemm_work, attn_smem(pd.Qmax));
    w = std::max(w, (size_t)NT * D * 16 + 4 * (size_t)(U * d.H + 16) + 256);
    w = std::max(w, sizeof(float) * 2 * (size_t)P * M);
    return w;
  };
  cudaDeviceProp prop;
  CUDA_TRY(cudaGetDeviceProperties(&prop, h->device));
  const size_t limit = prop.sharedMemPerBlockOptin;
  auto slots_left = [&](size_t w, size_t sl) { return off_ring + w > limit ? (size_t)0 : (limit - off_ring - w) / (sl + 128); };
  size_t slot = SLOT, work = work_for(SLOT);
  if (slots_left(work, SLOT) < 4) {
    const size_t w16 = work_for(SLOT / 2);
    if (slots_left(w16, SLOT / 2) >= 4 || slots_left(work, SLOT) < 2) slot = SLOT / 2, work = w16;
  }
  if (slots_left(work, slot) < 2) return fail(OWSM_DEC_ERR_LIMIT, "shared memory too small");
  {
    const size_t wco = (size_t)NT * D * 16 + 4 * (size_t)(U * d.H + 16) + 256 + 16384;
    if (slots_left(std::max(work, wco), slot) >= std::min<size_t>(slots_left(work, slot), 4)) work = std::max(work, wco);
  }
  const int nslot = (int)std::min<size_t>((limit - off_ring - work) / (slot + 128), slot == SLOT ? 6 : 8);
  pd.nslot = nslot;
  pd.slot = (int)slot;
  pd.apos = (int)(slot / (DK * 2));
  pd.off_pre = (int)off_pre;
  pd.off_sched = (int)off_sched;
  pd.off_rows = (int)off_rows;
  pd.inflight = std::min(nslot, (int)(65536 / slot));
  pd.off_out = (int)off_out;
  pd.off_ring = (int)off_ring;
  pd.sstride = (int)slot + 128;
  pd.off_work = (int)(off_ring + (size_t)nslot * pd.sstride);
  pd.work_bytes = (int)work;
  smem = (size_t)pd.off_work + work;
  if (!base) return OWSM_DEC_OK;
  // set-up writes: the whole carved area to zero (the state owsm_dec_plan's fresh allocations start in),
  // then the block tables
  CUDA_TRY(cudaMemset(base, 0, need));
  for (int gi = 0; gi < NGEMM; ++gi) {
    CUDA_TRY(cudaMemcpy(const_cast<int*>(pd.goff[gi]), off[gi].data(), off[gi].size() * 4, cudaMemcpyHostToDevice));
    if (!blk[gi].empty())
      CUDA_TRY(cudaMemcpy(const_cast<int*>(pd.gblk[gi]), blk[gi].data(), blk[gi].size() * 4, cudaMemcpyHostToDevice));
  }
  CUDA_TRY(cudaFuncSetAttribute(kernel_for(pd.NT), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)limit));
  int per_sm = 0;
  CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel_for(pd.NT), BLOCK, smem));
  if (per_sm < 1) return fail(OWSM_DEC_ERR_LIMIT, "the kernel does not fit an SM");
  // The memset and the pageable uploads above run on the legacy stream and may still be in flight when they
  // return; the call launches on the caller's stream, which need not be ordered after the legacy stream (a
  // non-blocking stream is not): wait for them here, at set-up.
  CUDA_TRY(cudaDeviceSynchronize());
  return OWSM_DEC_OK;
}

extern "C" {

int owsm_dec_step_static(OwsmDec* h, void* stream, int R, int S, int C, int T, const int64_t* tokens,
                         int64_t tok_stride, const int64_t* offset, int64_t off_stride, void* self_k, void* self_v,
                         const void* cross_k, const void* cross_v, const int32_t* enc_len, float* logits,
                         void* new_kv, int64_t* pred, const uint8_t* notime, int first_time, int last_time) {
  if (!h || !tokens || !offset || !self_k || !self_v || !cross_k || !cross_v || !logits || !new_kv)
    return fail(OWSM_DEC_ERR_ARG, "null argument");
  if (!aligned16(self_k) || !aligned16(self_v) || !aligned16(cross_k) || !aligned16(cross_v))
    return fail(OWSM_DEC_ERR_ARG, "K/V buffers must be 16-byte aligned");
  if (R < 1 || S < 1 || C < S || T < 1) return fail(OWSM_DEC_ERR_ARG, "bad call shape");
  if (R * S > STATIC_MAX_TOKENS)
    return fail(OWSM_DEC_ERR_LIMIT, "owsm_dec_step_static takes at most " + std::to_string(STATIC_MAX_TOKENS) +
                                        " tokens (rows x window) per call; use owsm_dec_plan + owsm_dec_step");
  if (h->device < 0 || h->device >= STATIC_MAX_DEVICES) return fail(OWSM_DEC_ERR_LIMIT, "device index too large");
  DeviceGuard guard(h->device);  // the handle's device is current for the symbol lookup and the launch
  std::lock_guard<std::mutex> lock(g_static_mu);
  StaticLayout& sl = g_static[h->device];
  if (sl.serial != h->serial || sl.R != R || sl.S != S || sl.C != C || sl.T != T) {
    // first call for this handle and shape on the device: find the array, check the shape fits, lay it out
    PlanDev pd{};
    size_t smem = 0, need = 0;
    int rc = static_layout(h, R, S, C, T, nullptr, pd, smem, need);
    if (rc) return rc;
    if (need > STATIC_SCRATCH_BYTES)
      return fail(OWSM_DEC_ERR_LIMIT, "this call needs " + std::to_string(need) + " bytes of scratch; the fixed area holds " +
                                          std::to_string(STATIC_SCRATCH_BYTES) + " (use owsm_dec_plan + owsm_dec_step)");
    if (!sl.base) {
      void* ptr = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&ptr, owsm_static_scratch);
      if (e != cudaSuccess) return fail(OWSM_DEC_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
      sl.base = reinterpret_cast<uint8_t*>(ptr);
    }
    sl.serial = 0;
    CUDA_TRY(cudaDeviceSynchronize());  // no earlier fixed-scratch call may still read the old layout
    rc = static_layout(h, R, S, C, T, sl.base, pd, smem, need);
    if (rc) return rc;
    sl.pd = pd;
    sl.smem = smem;
    sl.R = R; sl.S = S; sl.C = C; sl.T = T;
    sl.serial = h->serial;
  }
  PlanDev pd = sl.pd;
  pd.max_spin = h->max_spin;
  // the inter-CTA counters start every call at zero (a call that gave up may have left them set)
  CUDA_TRY(cudaMemsetAsync(pd.ctr, 0, 8 * sizeof(uint32_t), reinterpret_cast<cudaStream_t>(stream)));
  CallArgs a{};
  a.tok = tokens; a.tok_stride = tok_stride;
  a.off = offset; a.off_stride = off_stride;
  a.kc = reinterpret_cast<__half*>(self_k); a.vc = reinterpret_cast<__half*>(self_v);
  a.ck = reinterpret_cast<const __half*>(cross_k); a.cv = reinterpret_cast<const __half*>(cross_v);
  a.enc_len = enc_len;
  a.logits = logits; a.new_kv = reinterpret_cast<__half*>(new_kv);
  a.pred = pred; a.notime = notime; a.ft = first_time; a.lt = last_time;
  a.beam_mode = 0;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.gridDim = dim3(pd.P);
  cfg.blockDim = dim3(BLOCK);
  cfg.dynamicSmemBytes = sl.smem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel_for(pd.NT), pd, a));
  return OWSM_DEC_OK;
}

}  // extern "C"
