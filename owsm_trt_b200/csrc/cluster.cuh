// The cluster kernel: the same decoder call as decoder_kernel with three grid-wide exchanges per layer
// instead of eight. Included by decoder.cu (it reuses that file's GEMM, attention and output-stage code).
//
// Layout of the call. The grid is NCL clusters of 4 CTAs (one CTA per SM). Per layer:
//   S1  cluster (head h, row group rg): LN1 of the group's tokens -> the head's q/k/v rows (each CTA 48 of
//       the 192 rows, exchanged through distributed shared memory) -> masked self-attention of the group's
//       rows, split over the 4 CTAs by row or by position range, partial softmax states exchanged the same
//       way and combined in a fixed order -> the head's slice of the out-projection (each CTA a quarter of
//       the output features, K = 64) added into the next residual buffer.
//   S2  the same for cross-attention: LN2 -> the head's cross-query rows -> attention over the group's
//       utterances' encoder frames -> the head's slice of the cross-out projection.
//   S3  cluster c < NCL3 owns F / NCL3 hidden units: LN3 of all tokens -> its FFN1 rows (+ReLU), exchanged
//       -> its slice of FFN2 (K = F / NCL3) added into the next residual buffer.
// The residual stream is int64 fixed point (32 fraction bits) in three rotating buffers: a stage reads
// buffer k, adds its contributions into buffer k + 1 with integer atomics (exact, so the result does not
// depend on their order: the call stays bit-reproducible) and zeroes buffer k + 2, which the stage before
// read. Every CTA also adds its slice of (input residual + the stage's output bias), so each element of the
// next buffer is x + bias + the sum of the heads' (or hidden slices') contributions.
//
// Exchanges inside a cluster use st.async stores into the other CTAs' shared memory, counted in bytes on
// the receiver's mbarrier (which expects the bytes it will receive), so no cluster-wide barrier is needed
// after start-up and the producer warp never has to take part in one. All waits are bounded.
#pragma once

namespace owsm {

constexpr int CS = 4;          // CTAs per cluster
constexpr float kLog2e = 1.4426950408889634f;  // log2(e): the wide attention steps work in the log2 domain
constexpr int XQ_FLOATS = 16 * 3 * DK;  // exchange buffer: q/k/v rows of up to 16 tokens (fp32)
constexpr int PART_ENTRIES = 64;        // partial softmax states of one stage (units x queries)

// What this CTA's cluster owns in the three stages of a layer.
struct Cl {
  int cid, r;      // cluster index, rank in the cluster
  int h, rg;       // S1/S2: head and row group (valid when cid < H * RG)
  int u0, u1;      // utterances of the row group
  int b0, Rg;      // its rows
  int m0, Mg;      // its tokens [m0, m0 + Mg)
  bool ffn;        // S3: cid < NCL3
};

__device__ __forceinline__ Cl cluster_view(const PlanDev& pd) {
  Cl v;
  v.cid = blockIdx.x / CS;
  v.r = blockIdx.x % CS;
  const bool heads = v.cid < pd.H * pd.RG;
  v.h = heads ? v.cid % pd.H : 0;
  v.rg = heads ? v.cid / pd.H : 0;
  v.u0 = heads ? pd.U * v.rg / pd.RG : 0;
  v.u1 = heads ? pd.U * (v.rg + 1) / pd.RG : 0;
  v.b0 = v.u0 * pd.G;
  v.Rg = (v.u1 - v.u0) * pd.G;
  v.m0 = v.b0 * pd.S;
  v.Mg = v.Rg * pd.S;
  v.ffn = v.cid < pd.NCL3;
  return v;
}

// Attention units of a stage inside the cluster: `items` rows (S1) or utterances (S2), each split into
// `parts` position ranges when there are fewer items than CTAs; unit k = item * parts + part goes to
// cluster CTA k % 4.
__device__ __forceinline__ int unit_parts(int items) { return items >= CS ? 1 : CS / items; }

// Shared-memory view of the cluster stages' work area.
struct ClSmem {
  __half* bbuf;   // LayerNorm output, B-fragment order (NT tiles x D)
  float* xq;      // exchange: q/k/v (S1, [token][192]) or cross queries (S2, [token][64]) or FFN hidden
                  // (S3, B-fragment order over the cluster's F3 hidden units)
  float* part;    // exchange: partial softmax states [entry][XPS]
  __half* obuf;   // attention output of the group's tokens, B-fragment order (K = 64)
  uint8_t* attn;  // carve_attn area
};

__host__ __device__ constexpr size_t cl_bbuf_bytes(int NT, int D) { return (size_t)NT * D * 16; }
// The attention area doubles as the split-k partial sums of block_chunks (a warp's NT x 4 floats per lane).
__host__ __device__ constexpr size_t cl_attn_bytes(int NT, int Qmax) {
  return attn_smem(Qmax) > (size_t)NWARP * NT * 512 ? attn_smem(Qmax) : (size_t)NWARP * NT * 512;
}
__host__ __device__ constexpr size_t cl_work_bytes(int NT, int D, int Qmax) {
  return cl_bbuf_bytes(NT, D) + (size_t)XQ_FLOATS * 4 + (size_t)PART_ENTRIES * XPS * 4 + (size_t)4 * NT * 256 +
         cl_attn_bytes(NT, Qmax) + 64;
}

__device__ __forceinline__ ClSmem carve_cl(uint8_t* work, int NT, int D) {
  ClSmem s;
  uint8_t* p = work;
  s.bbuf = reinterpret_cast<__half*>(p); p += cl_bbuf_bytes(NT, D);
  s.xq = reinterpret_cast<float*>(p); p += (size_t)XQ_FLOATS * 4;
  s.part = reinterpret_cast<float*>(p); p += (size_t)PART_ENTRIES * XPS * 4;
  s.obuf = reinterpret_cast<__half*>(p); p += (size_t)4 * NT * 256;
  s.attn = p;
  return s;
}

// ------------------------------------------------------------------------------------------------ schedule
// Keys then values of positions p0 .. p1 - 1 (rows of 128 bytes), a chunk of at most apos positions each.
// keep: the rows are read by several clusters (an utterance's cross K/V in a beam call), so the copies do not
// mark them evict-first.
template <class Fn>
__device__ __forceinline__ void kv_chunks(const PlanDev& pd, const __half* kb, const __half* vb, int p0, int p1, Fn& fn,
                                          bool keep = false) {
  for (int j0 = p0; j0 < p1; j0 += pd.apos) {
    const int n = p1 - j0 < pd.apos ? p1 - j0 : pd.apos;
    fn((const void*)(kb + (long long)j0 * DK), (uint32_t)n * DK * 2, 1, 0u, keep);
    fn((const void*)(vb + (long long)j0 * DK), (uint32_t)n * DK * 2, 1, 0u, keep);
  }
}

// The byte ranges the producer copies for cluster stage `kind` of layer `l`, in the order the consumers use
// them: fn(src, piece_bytes, pieces, piece_stride_bytes, keep) per ring chunk (the pieces land back to back;
// keep: data other clusters read too, not evict-first).
template <class Fn>
__device__ void cl_chunks(const PlanDev& pd, const CallArgs& a, const Cl& cl, const int* pre, const int* offs,
                          int kind, int l, Fn&& fn) {
  const int D = pd.D, H = pd.H, S = pd.S, r = cl.r;
  auto blocks = [&](int gi, int blk) {  // one whole 16-row block (K = D) with its bias tail
    const GemmW& gw = pd.g[gi];
    fn((const void*)(gw.w + (long long)l * gw.lstride + (long long)blk * gw.bstride), (uint32_t)gw.bstride * 16, 1, 0u,
       false);
  };
  // 16-row blocks rb0 .. rb0 + nb - 1 of GEMM gi, k-blocks kb0 .. kb0 + nkb - 1 of each, packed per chunk
  auto kslices = [&](int gi, int rb0, int nb, int kb0, int nkb) {
    const GemmW& gw = pd.g[gi];
    const uint32_t piece = (uint32_t)nkb * 512;
    const int per = pd.slot / (int)piece;
    for (int b = 0; b < nb; b += per) {
      const int n = nb - b < per ? nb - b : per;
      fn((const void*)(gw.w + (long long)l * gw.lstride + (long long)(rb0 + b) * gw.bstride + (long long)kb0 * 32), piece,
         n, (uint32_t)gw.bstride * 16, false);
    }
  };
  if (kind == 1 || kind == 2) {
    if (cl.cid >= H * pd.RG || cl.Mg == 0) return;
    const int h = cl.h;
    if (kind == 1) {
      for (int j = 0; j < 3; ++j) {  // rows 48 r .. 48 r + 47 of the head's q | k | v
        const int i = 3 * r + j, part = i / 4, sub = i % 4;
        blocks(G_QKV, part * (D / 16) + 4 * h + sub);
      }
      const int parts = unit_parts(cl.Rg);
      for (int k = r; k < cl.Rg * parts; k += CS) {
        const int b = cl.b0 + k / parts, p = k % parts, off = offs[b];
        const long long base = (((long long)l * pd.Rs + b) * H + h) * pd.C * DK;
        kv_chunks(pd, a.kc + base, a.vc + base, off * p / parts, off * (p + 1) / parts, fn);
      }
      kslices(G_WO, r * (D / 64), D / 64, 4 * h, 4);
    } else {
      blocks(G_CQ, 4 * h + r);
      const int ng = cl.u1 - cl.u0, parts = unit_parts(ng);
      for (int k = r; k < ng * parts; k += CS) {
        const int u = cl.u0 + k / parts, p = k % parts, len = pre[u + 1] - pre[u];
        const long long base = (((long long)l * pd.Us + kv_utt(pd, u)) * H + h) * (long long)pd.T * DK;
        kv_chunks(pd, a.ck + base, a.cv + base, len * p / parts, len * (p + 1) / parts, fn, pd.kvg > 1);
      }
      kslices(G_WCO, r * (D / 64), D / 64, 4 * h, 4);
    }
    return;
  }
  if (kind == 3) {
    if (!cl.ffn) return;
    const int F3 = pd.F3, rows = F3 / CS;
    for (int j = 0; j < rows / 16; ++j) blocks(G_F1, (cl.cid * F3 + r * rows) / 16 + j);
    kslices(G_F2, r * (D / 64), D / 64, cl.cid * F3 / 16, F3 / 16);
  }
  (void)S;
}

}  // namespace owsm

namespace owsm {

// ------------------------------------------------------------------------------------------------ GEMM cores
// One 16-row block (A fragments at `ash` + lane * 16, nkb k-blocks, nkb even) times the B operand at `bsh`.
// The dependent mma chain, not the loads, sets a block's time, so the k-blocks go round four accumulator
// chains when nkb is a multiple of 4 (two otherwise).
template <int NT>
__device__ __forceinline__ void block_mma(uint32_t ash, int nkb, uint32_t bsh, float (&acc)[NT][4]) {
  const int lane = threadIdx.x & 31;
  float a1[NT][4], a2[NT][4], a3[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = a1[nt][e] = a2[nt][e] = a3[nt][e] = 0.f;
  uint32_t bp = bsh + lane * 8;
  if ((nkb & 3) == 0) {
#pragma unroll 1
    for (int kb = 0; kb < nkb; kb += 4) {
      const uint4 x0 = lds128_u32(ash + kb * 512);
      const uint4 x1 = lds128_u32(ash + (kb + 1) * 512);
      const uint4 x2 = lds128_u32(ash + (kb + 2) * 512);
      const uint4 x3 = lds128_u32(ash + (kb + 3) * 512);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint2 b0 = lds64_u32(bp + nt * 256);
        const uint2 b1 = lds64_u32(bp + (NT + nt) * 256);
        const uint2 b2 = lds64_u32(bp + (2 * NT + nt) * 256);
        const uint2 b3 = lds64_u32(bp + (3 * NT + nt) * 256);
        mma16816(acc[nt], x0, b0.x, b0.y);
        mma16816(a1[nt], x1, b1.x, b1.y);
        mma16816(a2[nt], x2, b2.x, b2.y);
        mma16816(a3[nt], x3, b3.x, b3.y);
      }
      bp += 4 * NT * 256;
    }
  } else {
#pragma unroll 2
    for (int kb = 0; kb < nkb; kb += 2) {
      const uint4 x0 = lds128_u32(ash + kb * 512);
      const uint4 x1 = lds128_u32(ash + (kb + 1) * 512);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint2 b0 = lds64_u32(bp + nt * 256);
        const uint2 b1 = lds64_u32(bp + (NT + nt) * 256);
        mma16816(acc[nt], x0, b0.x, b0.y);
        mma16816(a1[nt], x1, b1.x, b1.y);
      }
      bp += 2 * NT * 256;
    }
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] += (a1[nt][e] + a2[nt][e]) + a3[nt][e];
}

// All consumer warps on one ring chunk of `nblk` blocks (block i at abase + i * astride): warp w takes
// the blocks i with (first + i) % 7 == w, so a stage whose blocks span several chunks (first = the chunk's
// first block) spreads them evenly; epi(i, acc) per block.
template <int NT, class Epi>
__device__ __forceinline__ void chunk_gemm(uint32_t abase, int nblk, uint32_t astride, int nkb, uint32_t bsh, Epi&& epi,
                                           int first = 0) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = (warp - first % NWARP + NWARP) % NWARP; i < nblk; i += NWARP) {
    float acc[NT][4];
    block_mma<NT>(abase + (uint32_t)i * astride + lane * 16, nkb, bsh, acc);
    epi(i, acc);
  }
}

// The stage's single-block chunks j = 0 .. nch - 1 (16 rows x nkb k-blocks + a 64-byte bias tail), one warp
// per chunk: the warp whose index is the chunk's ring slot (warps past the slot count idle), so each slot has
// one consumer per phase. epi(j, acc, bias of rows g, g + 8).
// With at most half as many chunks as warps (and `red`, a shared-memory area of NWARP x NT x 512 bytes,
// given), a chunk's k-blocks are split over a team of NWARP / nch warps instead: a block's dependent mma
// chain, not the data, sets its time, so a team finishes it in a fraction of one warp's time. The team's
// other warps leave their partial sums in `red` and the first warp adds them up (in warp order) and runs epi.
template <int NT, class Epi>
__device__ void block_chunks(Ring& ring, int nch, int nkb, uint32_t bsh, Epi&& epi, float* red = nullptr,
                             const Ctx* cx = nullptr) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2;
  const int ns = ring.ns;
  if (red != nullptr && nch > 0 && 2 * nch <= NWARP && nch <= ns) {
    const int ts = NWARP / nch, j = warp / ts, w = warp % ts;
    if (j < nch) {
      // whole groups of 4 k-blocks where nkb allows (block_mma's four-chain form), else pairs
      const int u = (nkb & 3) == 0 ? 4 : 2, units = nkb / u, k0 = u * (units * w / ts), k1 = u * (units * (w + 1) / ts);
      const uint8_t* slot = ring.wait_at(ring.i + j);
      if (cx) event(*cx, 90);
      float acc[NT][4];
      block_mma<NT>(smem_u32(slot) + lane * 16 + (uint32_t)k0 * 512, k1 - k0, bsh + (uint32_t)k0 * NT * 256, acc);
      if (cx) event(*cx, 91);
      float bia[2] = {0.f, 0.f};
      if (w == 0) {
        const float* tail = reinterpret_cast<const float*>(slot + (size_t)nkb * 512);
        bia[0] = tail[g];
        bia[1] = tail[g + 8];
      }
      ring.release_at(ring.i + j, w == 0 ? NWARP - ts + 1 : 1);
      float* mine = red + (warp * 32 + lane) * (NT * 4);
      if (w > 0) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) sts128f(mine + nt * 4, make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]));
      }
      asm volatile("bar.sync %0, %1;" ::"r"(2 + j), "r"(ts * 32) : "memory");
      if (cx) event(*cx, 92);
      if (w == 0) {
        for (int o = 1; o < ts; ++o)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const float4 p = lds128f(mine + (o * 32) * (NT * 4) + nt * 4);
            acc[nt][0] += p.x;
            acc[nt][1] += p.y;
            acc[nt][2] += p.z;
            acc[nt][3] += p.w;
          }
        epi(j, acc, bia);
        if (cx) event(*cx, 93);
      }
    }
    ring.i += nch;
    return;
  }
  const int j0 = warp < ns ? (warp - (int)(ring.i % (uint32_t)ns) + ns) % ns : nch;
  for (int j = j0; j < nch; j += ns) {
    const uint8_t* slot = ring.wait_at(ring.i + j);
    float acc[NT][4];
    block_mma<NT>(smem_u32(slot) + lane * 16, nkb, bsh, acc);
    const float* tail = reinterpret_cast<const float*>(slot + (size_t)nkb * 512);
    const float bia[2] = {tail[g], tail[g + 8]};
    ring.release_at(ring.i + j);
    epi(j, acc, bia);
  }
  ring.i += nch;
}

// ------------------------------------------------------------------------------------------------ attention
// Online-softmax state of one warp for up to QM queries: running max and sum (warp-uniform) and two output
// dims per lane (2 lane, 2 lane + 1).
template <int QM>
struct WarpSoftmax {
  float m[QM], l[QM], o0[QM], o1[QM];
};

// One step of 8 key positions for one warp: lane (group g = lane / 4, quarter) scores position g over the
// 16 dims of its quarter (rotated by g, so the 8 rows of a step spread over the banks), the 4 lanes of a
// group add up, then every lane updates the state and accumulates the 8 value rows' dims 2 lane, 2 lane + 1.
// K / V rows: fp16 (`kh`, `vh`, 64 halves per row) or fp32 (`kf`, `vf`); n valid positions (<= 8); query q
// sees position i of the step when causal_base < 0 or causal_base + i <= q.
template <int QM, bool F32>
__device__ __forceinline__ void warp_step(WarpSoftmax<QM>& st, const float* qs, int Q, const void* kp, const void* vp,
                                          int n, int causal_base) {
  const int lane = threadIdx.x & 31, g = lane >> 2, part = ((lane & 3) + g) & 3;
  float kv[16];
  if (g < n) {
    if (F32) {
      const float* kr = reinterpret_cast<const float*>(kp) + g * DK + part * 16;
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        const float4 v = lds128f(kr + i);
        kv[i] = v.x; kv[i + 1] = v.y; kv[i + 2] = v.z; kv[i + 3] = v.w;
      }
    } else {
      const uint32_t ka = smem_u32(reinterpret_cast<const __half*>(kp) + g * DK + part * 16);
      const uint4 k0 = lds128_u32(ka), k1 = lds128_u32(ka + 16);
      const __half2* h0 = reinterpret_cast<const __half2*>(&k0);
      const __half2* h1 = reinterpret_cast<const __half2*>(&k1);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f0 = __half22float2(h0[e]), f1 = __half22float2(h1[e]);
        kv[2 * e] = f0.x; kv[2 * e + 1] = f0.y; kv[8 + 2 * e] = f1.x; kv[9 + 2 * e] = f1.y;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) kv[i] = 0.f;
  }
  // this step's value dims of the lane: rows 0 .. n - 1
  float2 vv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i < n) {
      if (F32) vv[i] = *reinterpret_cast<const float2*>(reinterpret_cast<const float*>(vp) + i * DK + 2 * lane);
      else {
        uint32_t raw;
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(raw) : "r"(smem_u32(reinterpret_cast<const __half*>(vp) + i * DK + 2 * lane)));
        vv[i] = __half22float2(*reinterpret_cast<__half2*>(&raw));
      }
    } else {
      vv[i] = make_float2(0.f, 0.f);
    }
  }
#pragma unroll
  for (int q = 0; q < QM; ++q) {
    if (q >= Q) break;
    const float* qq = qs + q * DK + part * 16;
    float sc = 0.f;
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
      const float4 a = lds128f(qq + i);
      sc += a.x * kv[i] + a.y * kv[i + 1] + a.z * kv[i + 2] + a.w * kv[i + 3];
    }
    sc += __shfl_xor_sync(0xffffffffu, sc, 1);
    sc += __shfl_xor_sync(0xffffffffu, sc, 2);
    const bool ok = g < n && (causal_base < 0 || causal_base + g <= q);
    if (!ok) sc = -INFINITY;
    float mx = sc;
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    const float mnew = fmaxf(st.m[q], mx);
    if (mnew == -INFINITY) continue;  // nothing visible yet
    const float al = st.m[q] > -INFINITY ? expf(st.m[q] - mnew) : 0.f;
    const float p = ok ? expf(sc - mnew) : 0.f;
    float ps = p;
    ps += __shfl_xor_sync(0xffffffffu, ps, 4);
    ps += __shfl_xor_sync(0xffffffffu, ps, 8);
    ps += __shfl_xor_sync(0xffffffffu, ps, 16);
    st.l[q] = st.l[q] * al + ps;
    float a0 = st.o0[q] * al, a1 = st.o1[q] * al;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float pi = __shfl_sync(0xffffffffu, p, i * 4);
      a0 += pi * vv[i].x;
      a1 += pi * vv[i].y;
    }
    st.o0[q] = a0;
    st.o1[q] = a1;
    st.m[q] = mnew;
  }
}

// Warp-wide maximum of a float (one instruction on sm_100a).
__device__ __forceinline__ float warp_max(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

// The permuted query layout of the wide steps: the two 16-byte halves of dims 8 c .. 8 c + 7 at float
// offsets 4 c and 32 + 4 c, so the lanes of a quarter warp, which read different chunks c of one half, hit
// different banks.
__device__ __forceinline__ int qperm(int d) { return ((d >> 2) & 1) * 32 + (d >> 3) * 4 + (d & 3); }

// One step of up to 32 key positions for one warp and one query, for long position ranges: lane i holds the
// whole key row of position i (64 dims in 32 half2 registers, its 16-byte pieces rotated by the lane so the
// rows of a quarter warp spread over the banks) and scores it against the query (permuted layout `qp`) in
// the log2 domain; the warp's max is one redux, the running sum of probabilities stays per lane (st.l, added
// up over the warp once the unit is done); the probabilities go through the warp's 32-float buffer and lane
// l adds up output dims 2 l, 2 l + 1 over the step's value rows, 8 rows per round. The query sees position
// i when causal_base < 0 or causal_base + i <= 0.
template <bool F32>
__device__ __forceinline__ void warp_step32(WarpSoftmax<1>& st, const float* qp, const void* kp, const void* vp, int n,
                                            int causal_base, float* pbuf) {
  const int lane = threadIdx.x & 31;
  uint32_t kr[32];
  if (lane < n) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int pc = (c + lane) & 7;
      if (F32) {
        const float* kf = reinterpret_cast<const float*>(kp) + lane * DK + pc * 8;
        const float4 u = lds128f(kf), w = lds128f(kf + 4);
        kr[4 * c] = pack_half2(u.x, u.y); kr[4 * c + 1] = pack_half2(u.z, u.w);
        kr[4 * c + 2] = pack_half2(w.x, w.y); kr[4 * c + 3] = pack_half2(w.z, w.w);
      } else {
        const uint4 u = lds128_u32(smem_u32(reinterpret_cast<const __half*>(kp) + lane * DK + pc * 8));
        kr[4 * c] = u.x; kr[4 * c + 1] = u.y; kr[4 * c + 2] = u.z; kr[4 * c + 3] = u.w;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) kr[i] = 0u;
  }
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int pc = (c + lane) & 7;
    const float4 a = lds128f(qp + pc * 4), b = lds128f(qp + 32 + pc * 4);
    const float2 k0 = unpack_half2(kr[4 * c]), k1 = unpack_half2(kr[4 * c + 1]);
    const float2 k2 = unpack_half2(kr[4 * c + 2]), k3 = unpack_half2(kr[4 * c + 3]);
    s0 = fmaf(a.x, k0.x, fmaf(a.y, k0.y, s0));
    s1 = fmaf(a.z, k1.x, fmaf(a.w, k1.y, s1));
    s2 = fmaf(b.x, k2.x, fmaf(b.y, k2.y, s2));
    s3 = fmaf(b.z, k3.x, fmaf(b.w, k3.y, s3));
  }
  const bool ok = lane < n && (causal_base < 0 || causal_base + lane <= 0);
  const float sc = ok ? ((s0 + s1) + (s2 + s3)) * kLog2e : -INFINITY;  // log2 domain
  const float mnew = fmaxf(st.m[0], warp_max(sc));
  if (mnew == -INFINITY) return;
  const float al = exp2f(st.m[0] - mnew);  // 0 while nothing was visible (m = -inf)
  const float p = ok ? exp2f(sc - mnew) : 0.f;
  st.l[0] = st.l[0] * al + p;
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(smem_u32(pbuf + lane)), "f"(p) : "memory");
  __syncwarp();
  float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
  // 8 value rows per round, loads issued together; rows past n have p = 0 and are not read
#pragma unroll 1
  for (int i0 = 0; i0 < n; i0 += 8) {
    const float4 pa = lds128f(pbuf + i0), pb = lds128f(pbuf + i0 + 4);
    const float pv[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
    float2 vv[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int i = i0 + e;
      if (F32) {
        vv[e] = i < n ? *reinterpret_cast<const float2*>(reinterpret_cast<const float*>(vp) + i * DK + 2 * lane) : make_float2(0.f, 0.f);
      } else {
        uint32_t r0 = 0u;
        if (i < n) asm volatile("ld.shared.u32 %0, [%1];" : "=r"(r0) : "r"(smem_u32(reinterpret_cast<const __half*>(vp) + i * DK + 2 * lane)));
        vv[e] = unpack_half2(r0);
      }
    }
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      a0 = fmaf(pv[e], vv[e].x, a0); a1 = fmaf(pv[e], vv[e].y, a1);
      b0 = fmaf(pv[e + 1], vv[e + 1].x, b0); b1 = fmaf(pv[e + 1], vv[e + 1].y, b1);
    }
  }
  __syncwarp();
  st.o0[0] = st.o0[0] * al + (a0 + b0);
  st.o1[0] = st.o1[0] * al + (a1 + b1);
  st.m[0] = mnew;
}


// One attention unit on all consumer warps, split-K inside the CTA: Q queries (s.q, fp32 [Q][64], scaled)
// over the cached keys/values of positions p0 .. p1 - 1 (ring chunks: keys then values, apos positions per
// chunk; warp w takes the steps of 8 positions w, w + 7, ... of each chunk and keeps its own online-softmax
// state, so no block barrier is needed per chunk), then with nnew > 0 the call's own keys/values (s.knew /
// s.vnew [nnew][64], fp32; query q sees new key j <= q, Q = nnew) on the warp with the least chunk work.
// The warps' states are merged once into the unit's partial state, handed to emit(q, c4, piece) as 17
// 16-byte pieces per query (unnormalised output dims, then the max in natural-log units and the sum);
// no barrier follows, so the caller passes one before it reads what emit stored. Wide units (WIDE, one
// query) read the query from s.out in the permuted layout of qperm, which the caller writes beside s.q.
template <int QM, bool WIDE, class Emit>
__device__ void attn_unit(const AttnSmem& s, Ring& ring, int Q, int p0, int p1, int apos, int nnew, const Ctx& cx,
                          Emit&& emit) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // long ranges of one query: steps of 32 positions (log2 domain); otherwise steps of 8 (the wide step's
  // registers would crowd the per-query state of several queries)
  const bool wide = WIDE && QM == 1 && p1 - p0 >= 256;
  WarpSoftmax<QM> st;
#pragma unroll
  for (int q = 0; q < QM; ++q) st.m[q] = -INFINITY, st.l[q] = 0.f, st.o0[q] = 0.f, st.o1[q] = 0.f;
  // this warp's probabilities of a wide step (after the merge's per-warp m, l; 16-byte aligned: the step
  // reads them with 128-bit loads)
  float* pbuf = s.sc + ((2 * NWARP * QM + 3) & ~3) + warp * 32;
  csync();  // the queries (and new keys / values) are in shared memory
  event(cx, 80);
  int last_steps = 0;
  for (int j0 = p0; j0 < p1; j0 += apos) {
    const int npos = p1 - j0 < apos ? p1 - j0 : apos;
    const __half* kt = reinterpret_cast<const __half*>(ring.wait_at(ring.i));
    const __half* vt = reinterpret_cast<const __half*>(ring.wait_at(ring.i + 1));
    if constexpr (WIDE && QM == 1) {
      if (wide) {
      // steps numbered across the whole unit (chunks hold whole steps), so the warps stay balanced when a
      // chunk's step count is not a multiple of the warp count
      const int nsteps = (npos + 31) >> 5, sbase = (j0 - p0) >> 5;
      for (int t = (warp - sbase % NWARP + NWARP) % NWARP; t < nsteps; t += NWARP) {
        const int n = npos - t * 32 < 32 ? npos - t * 32 : 32;
        warp_step32<false>(st, s.out, kt + (size_t)t * 32 * DK, vt + (size_t)t * 32 * DK, n, -1, pbuf);
      }
      last_steps = sbase + nsteps;
      }
    }
    if (!wide) {
      const int nsteps = (npos + 7) >> 3;
      for (int t = warp; t < nsteps; t += NWARP) {
        const int n = npos - t * 8 < 8 ? npos - t * 8 : 8;
        warp_step<QM, false>(st, s.q, Q, kt + (size_t)t * 8 * DK, vt + (size_t)t * 8 * DK, n, -1);
      }
      last_steps = nsteps;
    }
    __syncwarp();
    ring.release();  // keys
    ring.release();  // values
  }
  event(cx, 81);
  if (nnew > 0 && warp == (last_steps % NWARP)) {  // a warp with no more chunk steps than the others
    if constexpr (WIDE && QM == 1) {
      if (wide) warp_step32<true>(st, s.out, s.knew, s.vnew, nnew, 0, pbuf);  // nnew = 1 (one query)
    }
    if (!wide) {
      for (int j = 0; j < nnew; j += 8)
        warp_step<QM, true>(st, s.q, Q, s.knew + (size_t)j * DK, s.vnew + (size_t)j * DK, nnew - j < 8 ? nnew - j : 8, j);
    }
  }
  event(cx, 82);
  if constexpr (WIDE && QM == 1) {
    if (wide) {  // the lanes' running sums -> the warp's
#pragma unroll
      for (int o = 16; o; o >>= 1) st.l[0] += __shfl_xor_sync(0xffffffffu, st.l[0], o);
    }
  }
  // merge the warps: per warp m, l (sc area) and its output dims (scratch)
  float* wm = s.sc;
  float* wl = s.sc + NWARP * QM;
#pragma unroll
  for (int q = 0; q < QM; ++q) {
    if (q >= Q) break;
    if (lane == 0) {
      wm[warp * QM + q] = st.m[q];
      wl[warp * QM + q] = st.l[q];
    }
    *reinterpret_cast<float2*>(&s.scratch[(warp * Q + q) * DK + 2 * lane]) = make_float2(st.o0[q], st.o1[q]);
  }
  csync();
  // per query 17 pieces of 4 floats: dims 4 c4 .. 4 c4 + 3 (c4 < 16), then (max in natural-log units, sum)
  for (int idx = threadIdx.x; idx < Q * (XPS / 4); idx += NTHR) {
    const int q = idx / (XPS / 4), c4 = idx % (XPS / 4);
    float mx = -INFINITY;
    for (int w = 0; w < NWARP; ++w) mx = fmaxf(mx, wm[w * QM + q]);
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    float l = 0.f;
    if (mx > -INFINITY)
      for (int w = 0; w < NWARP; ++w) {
        const float mw = wm[w * QM + q];
        if (mw > -INFINITY) {
          const float f = wide ? exp2f(mw - mx) : expf(mw - mx);
          if (c4 < DK / 4) {
            const float4 sv = lds128f(&s.scratch[(w * Q + q) * DK + c4 * 4]);
            o.x += f * sv.x;
            o.y += f * sv.y;
            o.z += f * sv.z;
            o.w += f * sv.w;
          } else {
            l += f * wl[w * QM + q];
          }
        }
      }
    emit(q, c4, c4 < DK / 4 ? o : make_float4(wide ? mx / kLog2e : mx, l, 0.f, 0.f));
  }
}

// ------------------------------------------------------------------------------------------------ stages
// Embedding into the fixed-point residual buffer 0 (this CTA's slice); buffer 1, which the first stage adds
// into, is zeroed.
__device__ void cl_embed(const PlanDev& pd, const CallArgs& a, const Ctx& cx, int c) {
  const long long total = (long long)pd.M * pd.D;
  const long long lo = total * c / pd.P, hi = total * (c + 1) / pd.P;
  for (long long i = lo + threadIdx.x; i < hi; i += NTHR) {
    const int m = (int)(i / pd.D), n = (int)(i % pd.D);
    const int r = m / pd.S, s = m % pd.S;
    long long t = a.tok[(long long)r * a.tok_stride + s];
    t = t < 0 ? 0 : (t >= pd.V ? pd.V - 1 : t);
    long long pos = (long long)cx.offs[r] + s;
    pos = pos >= pd.max_pos ? pd.max_pos - 1 : pos;
    pd.xf[0][i] = to_fix(__half2float(pd.emb[t * pd.D + n]) * pd.xscale + pd.pe[pos * pd.D + n]);
    pd.xf[1][i] = 0;
  }
}

// This CTA's slice of the next residual buffer: + input residual + the stage's output bias; and its slice
// of the free buffer zeroed (the stage after next adds into it).
// Part c of n of the pass (the stage's idle CTAs share it when it has any, so the CTAs with work start their
// LayerNorm at once; otherwise all P CTAs).
__device__ void cl_residual(const PlanDev& pd, int gi, int l, const long long* xin, long long* xout, long long* xfree,
                            int c, int n) {
  const long long total = (long long)pd.M * pd.D;
  const long long lo = total * c / n, hi = total * (c + 1) / n;
  const float* bias = pd.g[gi].b + (long long)l * pd.D;
  // 4 elements per thread per round, loads first: one L2 round trip per round, not per element
  for (long long i0 = lo + threadIdx.x; i0 < hi; i0 += 4 * NTHR) {
    long long v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const long long i = i0 + (long long)e * NTHR;
      if (i < hi) v[e] = __ldcg(xin + i) + to_fix(__ldg(bias + i % pd.D));
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const long long i = i0 + (long long)e * NTHR;
      if (i < hi) {
        red_add_s64(xout + i, v[e]);
        xfree[i] = 0;
      }
    }
  }
}

// LayerNorm of tokens 0 .. M - 1 (residual rows m0 ..) into the B operand at bbuf, the same on every CTA of
// the cluster. From CL_LN_SPLIT tokens on, each CTA normalises a quarter of them (a row costs the loads'
// round trips, not bandwidth, so four CTAs finish in about the time of one quarter) and stores their
// fragments into the other CTAs' bbuf through st.async on the exchange barrier xb; the CTAs' tokens are
// disjoint, so each B operand is the one a single CTA would have made. Ends with the operand complete.
// The LayerNorm itself runs out of line: inlined into every stage of the cluster kernel, its 32 registers of
// row values pushed the kernel's allocation into spills across the GEMM and attention loops (a called copy
// measured about 7% faster at batch 1 and 19% at batch 16; the grid-stage kernel keeps it inline, where the
// call measured slower).
// The padding tokens' fragments are left as they are: a GEMM's output column m depends on B column m alone,
// and every epilogue of this kernel drops the columns of padding tokens.
__device__ __noinline__ void cl_ln_call(const PlanDev& pd, const long long* x, int m0, int M, int NT, __half* bbuf,
                                        const Ctx& cx, int r0, int r1) {
  ln_rows(pd, x, m0, M, NT, bbuf, cx, r0, r1, false);
}

constexpr int CL_LN_SPLIT = 8;
__device__ void cl_ln_rows(const PlanDev& pd, const long long* x, int m0, int M, int NT, __half* bbuf, const Ctx& cx,
                           int r, uint64_t* xb, uint32_t& ph, Ring& ring) {
  const bool split = M >= CL_LN_SPLIT;
  const int D = pd.D, r0 = split ? M * r / CS : 0, r1 = split ? M * (r + 1) / CS : M;
  if (split && threadIdx.x == 0) mbar_arrive_expect_tx(xb, (uint32_t)((M - (r1 - r0)) * D * 2));
  cl_ln_call(pd, x, m0, M, NT, bbuf, cx, r0, r1);
  csync();
  if (!split) return;
  // a token's fragments: per k-block 32 contiguous bytes, k-blocks NT * 256 bytes apart
  const uint32_t b_s = smem_u32(bbuf), xb_s = smem_u32(xb);
  const int per_row = D / 8;  // 16-byte pieces of a token
  for (int i = threadIdx.x; i < (r1 - r0) * per_row; i += NTHR) {
    const int m = r0 + i / per_row, c = i % per_row;
    const uint32_t off = (uint32_t)((((c >> 1) * NT + (m >> 3)) * 32 + (m & 7) * 4) * 8 + (c & 1) * 16);
    const uint4 v = lds128_u32(b_s + off);
#pragma unroll
    for (int q = 1; q < CS; ++q) {
      const uint32_t dst = (uint32_t)((r + q) % CS);
      st_async_v4(mapa_shared(b_s + off, dst), v, mapa_shared(xb_s, dst));
    }
  }
  if (!mbar_wait_cluster(xb, ph, pd.max_spin)) {
    ring.dead = true;
    atomicExch(pd.err, E_ERR_TIMEOUT);
  }
  ph ^= 1u;
}

// Four consecutive fp16 values (exact: v holds fp16-rounded values) at p: one 8-byte store where p allows.
__device__ __forceinline__ void store4h(__half* p, const float4& v) {
  const __half2 lo = __floats2half2_rn(v.x, v.y), hi = __floats2half2_rn(v.z, v.w);
  if ((reinterpret_cast<uintptr_t>(p) & 7) == 0) {
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&lo);
    u.y = *reinterpret_cast<const uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(p) = u;
  } else {
    p[0] = __low2half(lo);
    p[1] = __high2half(lo);
    p[2] = __low2half(hi);
    p[3] = __high2half(hi);
  }
}

// S1 (kind 1, self-attention) or S2 (kind 2, cross-attention) of a cluster that owns (head h, row group).
// QM: compile-time bound of the queries of an attention unit (1 for one-token calls without row sharing).
template <int NT, int QM, bool WIDE>
__device__ void cl_attn_stage(const PlanDev& pd, const CallArgs& a, Ring& ring, const Ctx& cx, const Cl& cl,
                              const int* pre, int kind, int l, uint8_t* work, uint64_t* xbar, uint32_t (&ph)[3],
                              const long long* xin, long long* xout) {
  const int D = pd.D, H = pd.H, S = pd.S, h = cl.h, r = cl.r, Mg = cl.Mg;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const ClSmem sm = carve_cl(work, NT, D);
  const int nq = kind == 1 ? 3 * DK : DK;  // the head's projected rows: q | k | v, or q
  const int my = kind == 1 ? 48 : 16;      // of which this CTA computes rows my * r .. my * r + my - 1
  const int items = kind == 1 ? cl.Rg : cl.u1 - cl.u0;
  const int parts = unit_parts(items), nunits = items * parts;
  const int Qu = kind == 1 ? S : pd.G * S;  // queries of a unit
  const int mine = r < nunits ? (nunits - r + CS - 1) / CS : 0;
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&xbar[0], (uint32_t)((CS - 1) * my * Mg * 4));
    mbar_arrive_expect_tx(&xbar[1], (uint32_t)((nunits - mine) * Qu * XPS * 4));
  }
  cl_ln_rows(pd, xin, cl.m0, Mg, NT, sm.bbuf, cx, r, &xbar[2], ph[2], ring);
  event(cx, 51);
  const uint32_t xq_s = smem_u32(sm.xq), part_s = smem_u32(sm.part);
  const uint32_t bar0_s = smem_u32(&xbar[0]), bar1_s = smem_u32(&xbar[1]);
  // (the other CTAs' addresses are mapped where they are used: keeping them live through the stage costs
  // registers the attention code needs)
  // the head's projection rows of this CTA -> every cluster CTA's exchange buffer (and the cache)
  block_chunks<NT>(ring, my / 16, D / 16, smem_u32(sm.bbuf), [&](int j, const float (&acc)[NT][4], const float (&bia)[2]) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = my * r + j * 16 + g + (e >> 1) * 8, m = nt * 8 + 2 * t + (e & 1);
        if (m >= Mg) continue;
        // fp16 like the projection output the reference attends with
        sm.xq[m * nq + row] = __half2float(__float2half_rn(acc[nt][e] + bia[e >> 1]));
      }
  }, reinterpret_cast<float*>(sm.attn), &cx);
  csync();
  // this CTA's rows of each token, 4 at a time: to the other cluster CTAs' exchange buffers and, for key and
  // value rows (4 dims of one row: my and DK are multiples of 4), to the cache slot and new_kv
  const int pieces = my / 4;
  for (int i = threadIdx.x; i < Mg * pieces; i += NTHR) {
    const int m = i / pieces, row = my * r + (i % pieces) * 4, idx = m * nq + row;
    const float4 v = lds128f(&sm.xq[idx]);
    const uint4 w = make_uint4(__float_as_uint(v.x), __float_as_uint(v.y), __float_as_uint(v.z), __float_as_uint(v.w));
#pragma unroll
    for (int q = 1; q < CS; ++q) {
      const uint32_t dst = (uint32_t)((r + q) % CS);
      st_async_v4(mapa_shared(xq_s + idx * 4, dst), w, mapa_shared(bar0_s, dst));
    }
    if (kind == 1 && row >= DK) {
      const int mg = cl.m0 + m, b = mg / S, s = mg % S, kv = (row - DK) / DK, d = (row - DK) % DK;
      const long long cslot = ((((long long)l * pd.Rs + b) * H + h) * pd.C + cx.offs[b] + s) * DK + d;
      store4h((kv ? a.vc : a.kc) + cslot, v);
      store4h(a.new_kv + ((((long long)(l * 2 + kv) * pd.Rs + b) * H + h) * S + s) * DK + d, v);
    }
  }
  event(cx, 52);
  if (!mbar_wait_cluster(&xbar[0], ph[0], pd.max_spin)) {
    ring.dead = true;
    atomicExch(pd.err, E_ERR_TIMEOUT);
  }
  ph[0] ^= 1u;
  event(cx, 53);
  // this CTA's attention units -> their partial softmax states into every cluster CTA's table
  const AttnSmem as = carve_attn(sm.attn, pd.Qmax);
  for (int k = r; k < nunits; k += CS) {
    const int item = k / parts, p = k % parts;
    int p0, p1, nnew = 0;
    if (kind == 1) {
      const int b = cl.b0 + item, off = cx.offs[b];
      p0 = off * p / parts;
      p1 = off * (p + 1) / parts;
      nnew = (p == parts - 1) ? S : 0;
      for (int idx = threadIdx.x; idx < S * DK; idx += NTHR) {
        const int q = idx / DK, d = idx % DK, ml = item * S + q;
        as.q[idx] = sm.xq[ml * nq + d] * 0.125f;
        if (QM == 1 && WIDE) as.out[qperm(d)] = as.q[idx];  // the wide steps' copy (s.out until the merge)
        as.knew[idx] = sm.xq[ml * nq + DK + d];
        as.vnew[idx] = sm.xq[ml * nq + 2 * DK + d];
      }
    } else {
      const int u = cl.u0 + item, len = pre[u + 1] - pre[u];
      p0 = len * p / parts;
      p1 = len * (p + 1) / parts;
      for (int idx = threadIdx.x; idx < Qu * DK; idx += NTHR) {
        const int q = idx / DK, d = idx % DK;
        as.q[idx] = sm.xq[(item * Qu + q) * nq + d] * 0.125f;
        if (QM == 1 && WIDE) as.out[qperm(d)] = as.q[idx];
      }
    }
    // the unit's partial state -> this CTA's table and every other cluster CTA's
    attn_unit<QM, WIDE>(as, ring, Qu, p0, p1, pd.apos, nnew, cx, [&](int q, int c4, const float4& v) {
      const int off = (k * Qu + q) * XPS + c4 * 4;
      sts128f(&sm.part[off], v);
      const uint4 w = make_uint4(__float_as_uint(v.x), __float_as_uint(v.y), __float_as_uint(v.z), __float_as_uint(v.w));
#pragma unroll
      for (int i = 1; i < CS; ++i) {
        const uint32_t dst = (uint32_t)((r + i) % CS);
        st_async_v4(mapa_shared(part_s + off * 4, dst), w, mapa_shared(bar1_s, dst));
      }
    });
    event(cx, 54);
  }
  csync();  // this CTA's own entries are in the table (the next unit's staging needed none: it touches no
            // area the merge reads, and attn_unit starts with a barrier)
  if (!mbar_wait_cluster(&xbar[1], ph[1], pd.max_spin)) {
    ring.dead = true;
    atomicExch(pd.err, E_ERR_TIMEOUT);
  }
  ph[1] ^= 1u;
  event(cx, 55);
  // every token of the group: its units' parts combined in part order -> the out-projection's B operand
  // (padding tokens' columns are left as they are: the out-projection's epilogue drops them)
  for (int idx = threadIdx.x; idx < Mg * (DK / 2); idx += NTHR) {
    const int m = idx / (DK / 2), dp = idx % (DK / 2);
    float n0 = 0.f, n1 = 0.f;
    {
      const int item = m / Qu, q = m % Qu;
      const float* e0 = sm.part + ((size_t)(item * parts) * Qu + q) * XPS;
      const size_t step = (size_t)Qu * XPS;
      float mx = -INFINITY;
      for (int p = 0; p < parts; ++p) mx = fmaxf(mx, e0[p * step + DK]);
      float den = 0.f;
      for (int p = 0; p < parts; ++p) {
        const float mp = e0[p * step + DK];
        if (mp > -INFINITY) {
          const float w = expf(mp - mx);
          den += w * e0[p * step + DK + 1];
          n0 += w * e0[p * step + 2 * dp];
          n1 += w * e0[p * step + 2 * dp + 1];
        }
      }
      const float inv = den > 0.f ? 1.f / den : 0.f;
      n0 *= inv;
      n1 *= inv;
    }
    *reinterpret_cast<__half2*>(&sm.obuf[bfrag_idx(m, 2 * dp, NT)]) = __floats2half2_rn(n0, n1);
  }
  csync();
  event(cx, 56);
  // the head's slice of the out-projection: output rows (D / 4) r .. , k-blocks 4 h .. 4 h + 3
  const int nb = D / 64, per = pd.slot / 2048;
  for (int bb = 0; bb < nb; bb += per) {
    const int n = nb - bb < per ? nb - bb : per;
    const uint8_t* slot = ring.wait();
    chunk_gemm<NT>(smem_u32(slot), n, 2048u, 4, smem_u32(sm.obuf), [&](int i, const float (&acc)[NT][4]) {
      const int rb = r * nb + bb + i;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int nn = rb * 16 + g + (e >> 1) * 8, m = nt * 8 + 2 * t + (e & 1);
          if (m < Mg) red_add_s64(xout + (long long)(cl.m0 + m) * D + nn, to_fix(acc[nt][e]));
        }
    }, bb);
    ring.release();
  }
}

// S3: FFN1 rows of this cluster's hidden slice (+ReLU), exchanged as B fragments; FFN2 slice -> residual.
template <int NT>
__device__ void cl_ffn_stage(const PlanDev& pd, Ring& ring, const Ctx& cx, const Cl& cl, uint8_t* work,
                             uint64_t* xbar, uint32_t (&ph)[3], const long long* xin, long long* xout) {
  const int D = pd.D, M = pd.M, r = cl.r, F3 = pd.F3, rows = F3 / CS, nkb3 = F3 / 16;
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const ClSmem sm = carve_cl(work, NT, D);
  __half* hb = reinterpret_cast<__half*>(sm.xq);  // B fragments over the F3 hidden units (nkb3 k-blocks)
  const int kb_mine = rows / 16;                   // this CTA's k-blocks: r * kb_mine ..
  const uint32_t my_bytes = (uint32_t)kb_mine * NT * 256;
  if (threadIdx.x == 0) mbar_arrive_expect_tx(&xbar[0], (CS - 1) * my_bytes);
  cl_ln_rows(pd, xin, 0, M, NT, sm.bbuf, cx, r, &xbar[2], ph[2], ring);
  event(cx, 60);
  block_chunks<NT>(ring, rows / 16, D / 16, smem_u32(sm.bbuf), [&](int j, const float (&acc)[NT][4], const float (&bia)[2]) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int k = r * rows + j * 16 + g + (e >> 1) * 8, m = nt * 8 + 2 * t + (e & 1);
        const float y = m < M ? fmaxf(acc[nt][e] + bia[e >> 1], 0.f) : 0.f;
        hb[bfrag_idx(m, k, NT)] = __float2half_rn(y);
      }
  }, reinterpret_cast<float*>(sm.attn), &cx);
  csync();
  event(cx, 61);
  const uint32_t mine_s = smem_u32(hb) + (uint32_t)r * my_bytes;
  const uint32_t bar0 = smem_u32(&xbar[0]);
  for (int i = threadIdx.x; i < (int)(my_bytes / 16); i += NTHR) {
    const uint4 v = lds128_u32(mine_s + i * 16);
#pragma unroll
    for (int q = 1; q < CS; ++q) {
      const uint32_t dst = (uint32_t)((r + q) % CS);
      st_async_v4(mapa_shared(mine_s + i * 16, dst), v, mapa_shared(bar0, dst));
    }
  }
  if (!mbar_wait_cluster(&xbar[0], ph[0], pd.max_spin)) {
    ring.dead = true;
    atomicExch(pd.err, E_ERR_TIMEOUT);
  }
  ph[0] ^= 1u;
  event(cx, 63);
  const int nb = D / 64, piece = nkb3 * 512, per = pd.slot / piece;
  for (int bb = 0; bb < nb; bb += per) {
    const int n = nb - bb < per ? nb - bb : per;
    const uint8_t* slot = ring.wait();
    chunk_gemm<NT>(smem_u32(slot), n, (uint32_t)piece, nkb3, smem_u32(hb), [&](int i, const float (&acc)[NT][4]) {
      const int rb = r * nb + bb + i;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int nn = rb * 16 + g + (e >> 1) * 8, m = nt * 8 + 2 * t + (e & 1);
          if (m < M) red_add_s64(xout + (long long)m * D + nn, to_fix(acc[nt][e]));
        }
    }, bb);
    ring.release();
  }
}

}  // namespace owsm

namespace owsm {

// The output stage of the cluster kernel (greedy calls): final LayerNorm of the fixed-point residual,
// this CTA's vocab blocks (the grid kernel's block schedule), logits out and the running argmax per token
// (first index on ties; timestamp ids left out for flagged rows), merged over the warps into os.amax/aidx.
template <int NT>
__device__ void cl_out_stage(const PlanDev& pd, const CallArgs& a, Ring& ring, const Ctx& cx, uint8_t* work,
                             OutState& os, uint64_t* xb, uint32_t& ph) {
  const int M = pd.M, V = pd.V;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  __half* bbuf = reinterpret_cast<__half*>(work);
  if (a.rules)  // the timestamp-rule state of every token (read by the argmax after the next barrier)
    for (int m = threadIdx.x; m < M; m += NTHR) rule_state(pd, a, m, os.topi + m * KTOP);
  cl_ln_rows(pd, pd.xfix, 0, M, NT, bbuf, cx, (int)(blockIdx.x % CS), xb, ph, ring);
  event(cx, 70);
  float best[NT][2];
  int besti[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) best[nt][0] = best[nt][1] = -INFINITY, besti[nt][0] = besti[nt][1] = 0x7fffffff;
  const int b0 = cx.so[G_OUT];
  block_chunks<NT>(ring, cx.so[G_OUT + 1] - b0, pd.D / 16, smem_u32(bbuf),
                   [&](int j, const float (&acc)[NT][4], const float (&bia)[2]) {
                     const int rb = cx.sb[b0 + j];
#pragma unroll
                     for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                       for (int e = 0; e < 4; ++e) {
                         const int n = rb * 16 + g + (e >> 1) * 8, m = nt * 8 + 2 * t + (e & 1);
                         if (m >= M || n >= V) continue;
                         const float y = acc[nt][e] + bia[e >> 1];
                         a.logits[(long long)m * V + n] = y;
                         const float ya = argmax_bad(pd, a, os.topi + m * KTOP, m, n) ? -INFINITY : y;
                         merge_best(best[nt][e & 1], besti[nt][e & 1], ya, n);
                       }
                   });
  event(cx, 71);
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
  csync();
  for (int m = threadIdx.x; m < M; m += NTHR) {
    float bv = os.amax[m];
    int bi = os.aidx[m];
    for (int w = 0; w < NWARP; ++w) merge_best(bv, bi, os.wamax[w * M + m], os.waidx[w * M + m]);
    os.amax[m] = bv;
    os.aidx[m] = bi;
  }
  csync();
}

// (y, n) into a list of KTOP (value, id) in registers, sorted best first by beats(), if it beats the last
// entry: it takes the place of the first entry it beats and the entries from there on move down one place
// (the same list as inserting by shifting; the comparisons are independent of one another).
__device__ __forceinline__ void list_push(float (&v)[KTOP], int (&id)[KTOP], float y, int n) {
  bool b[KTOP];
#pragma unroll
  for (int e = 0; e < KTOP; ++e) b[e] = beats(y, n, v[e], id[e]);
#pragma unroll
  for (int e = KTOP - 1; e >= 0; --e)
    if (b[e]) {
      const bool sh = e > 0 && b[e - 1];
      v[e] = sh ? v[e - 1] : y;
      id[e] = sh ? id[e - 1] : n;
    }
}

// The output stage of a beam call: final LayerNorm, this CTA's vocab blocks, logits out, and per token the
// running max / sum of exp (log-softmax partials) and top-K over this CTA's ids, first per warp (a 16-row
// tile at a time, as the grid kernel does), then merged over the warps into os.rmax / rsum / topv / topi.
template <int NT>
__device__ void cl_out_stage_beam(const PlanDev& pd, const CallArgs& a, Ring& ring, const Ctx& cx, uint8_t* work,
                                  OutState& os, uint64_t* xb, uint32_t& ph) {
  const int M = pd.M, V = pd.V, K = pd.beam;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  __half* bbuf = reinterpret_cast<__half*>(work);
  cl_ln_rows(pd, pd.xfix, 0, M, NT, bbuf, cx, (int)(blockIdx.x % CS), xb, ph, ring);
  event(cx, 70);
  // Per lane and token (nt, s2) -- token nt * 8 + 2 t + s2, whose values in a block are vocabulary rows g and
  // g + 8, held by the 8 lanes g = 0 .. 7 of that t: the running max and sum of exp of the lane's values
  // (log-softmax partials), and entry g of the warp's sorted list of the token's KTOP best (value, id) so far
  // (one entry per lane; empty entries carry distinct ids, so every element of a merge has its own rank).
  float rmx[NT][2], rsm[NT][2], lv[NT][2];
  int li[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int s2 = 0; s2 < 2; ++s2)
      rmx[nt][s2] = lv[nt][s2] = -INFINITY, rsm[nt][s2] = 0.f, li[nt][s2] = 0x7fffffff - g;
  const int b0 = cx.so[G_OUT];
  block_chunks<NT>(ring, cx.so[G_OUT + 1] - b0, pd.D / 16, smem_u32(bbuf),
                   [&](int j, const float (&acc)[NT][4], const float (&bia)[2]) {
                     const int rb = cx.sb[b0 + j], n0 = rb * 16 + g, n1 = n0 + 8;
                     float y0s[2 * NT], y1s[2 * NT];
                     unsigned need = 0;  // bit k: token slot k = 2 nt + s2 has values for the list
#pragma unroll
                     for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                       for (int s2 = 0; s2 < 2; ++s2) {
                         const int m = nt * 8 + 2 * t + s2;
                         float y0 = acc[nt][s2] + bia[0], y1 = acc[nt][2 + s2] + bia[1];
                         if (m < M) {
                           if (n0 < V) a.logits[(long long)m * V + n0] = y0;
                           if (n1 < V) a.logits[(long long)m * V + n1] = y1;
                         }
                         if (m >= M || n0 >= V) y0 = -INFINITY;
                         if (m >= M || n1 >= V) y1 = -INFINITY;
                         const float mx = fmaxf(rmx[nt][s2], fmaxf(y0, y1));
                         if (mx > -INFINITY) {
                           float sm = rmx[nt][s2] > -INFINITY ? rsm[nt][s2] * expf(rmx[nt][s2] - mx) : 0.f;
                           if (y0 > -INFINITY) sm += expf(y0 - mx);
                           if (y1 > -INFINITY) sm += expf(y1 - mx);
                           rmx[nt][s2] = mx;
                           rsm[nt][s2] = sm;
                         }
                         // the token's K-th best so far (lane g = K - 1 of this t) bars the block's values
                         const float bv = __shfl_sync(0xffffffffu, lv[nt][s2], (K - 1) * 4 + t);
                         const int bi = __shfl_sync(0xffffffffu, li[nt][s2], (K - 1) * 4 + t);
                         const bool cand = m < M && (beats(y0, n0, bv, bi) || beats(y1, n1, bv, bi));
                         if (__any_sync(0xffffffffu, cand)) need |= 1u << (2 * nt + s2);
                         y0s[2 * nt + s2] = y0;
                         y1s[2 * nt + s2] = y1;
                       }
                     // the merges, one copy of the code for all slots (it runs once per call and SM, so its
                     // size, not only its instruction count, sets its time): the slot's values are moved in and
                     // out by predicated moves
#pragma unroll 1
                     for (int k = 0; k < 2 * NT; ++k) {
                       if (!((need >> k) & 1u)) continue;
                       const int m = (k >> 1) * 8 + 2 * t + (k & 1);
                       float ev[3] = {0.f, 0.f, 0.f};
                       int ei[3] = {0, n0, n1};
#pragma unroll
                       for (int kk = 0; kk < 2 * NT; ++kk)
                         if (kk == k) ev[0] = lv[kk >> 1][kk & 1], ei[0] = li[kk >> 1][kk & 1], ev[1] = y0s[kk], ev[2] = y1s[kk];
                       // merge: the rank of each of the lane's 3 elements among the token's 24 (8 lanes x
                       // {list entry, y0, y1}); the element of rank q < KTOP becomes entry q (lane q)
                       int rk[3] = {0, 0, 0};
#pragma unroll
                       for (int o = 0; o < 8; ++o) {
                         const int src = o * 4 + t;
#pragma unroll
                         for (int q = 0; q < 3; ++q) {
                           const float ov = __shfl_sync(0xffffffffu, ev[q], src);
                           const int oi = __shfl_sync(0xffffffffu, ei[q], src);
#pragma unroll
                           for (int e = 0; e < 3; ++e) rk[e] += beats(ov, oi, ev[e], ei[e]) ? 1 : 0;
                         }
                       }
                       float* tv = os.wtopv + ((size_t)warp * M + (m < M ? m : 0)) * KTOP;
                       int* ti = os.wtopi + ((size_t)warp * M + (m < M ? m : 0)) * KTOP;
#pragma unroll
                       for (int e = 0; e < 3; ++e)
                         if (m < M && rk[e] < KTOP) tv[rk[e]] = ev[e], ti[rk[e]] = ei[e];
                       __syncwarp();
                       const float nv = m < M ? tv[g] : 0.f;
                       const int ni = m < M ? ti[g] : 0;
                       __syncwarp();
#pragma unroll
                       for (int kk = 0; kk < 2 * NT; ++kk)
                         if (kk == k && m < M) lv[kk >> 1][kk & 1] = nv, li[kk >> 1][kk & 1] = ni;
                     }
                   });
  // the 8 lanes of a token (g = 0 .. 7) combine their partials; the warp's partial per token -> os.wrmax / wrsum;
  // its list -> os.wtopv / wtopi (entry g from lane g)
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int s2 = 0; s2 < 2; ++s2) {
      float mx = rmx[nt][s2], sm = rsm[nt][s2];
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        const float om = __shfl_xor_sync(0xffffffffu, mx, o), osm = __shfl_xor_sync(0xffffffffu, sm, o);
        const float nm = fmaxf(mx, om);
        if (nm > -INFINITY) {
          sm = (mx > -INFINITY ? sm * expf(mx - nm) : 0.f) + (om > -INFINITY ? osm * expf(om - nm) : 0.f);
          mx = nm;
        }
      }
      const int m = nt * 8 + 2 * t + s2;
      if (m < M) {
        if (g == 0) {
          os.wrmax[warp * M + m] = mx;
          os.wrsum[warp * M + m] = sm;
        }
        os.wtopv[((size_t)warp * M + m) * KTOP + g] = lv[nt][s2];
        os.wtopi[((size_t)warp * M + m) * KTOP + g] = li[nt][s2];
      }
    }
  event(cx, 71);
  csync();
  for (int m = threadIdx.x; m < M; m += NTHR) {
    float mx = os.rmax[m];
    for (int w = 0; w < NWARP; ++w) mx = fmaxf(mx, os.wrmax[w * M + m]);
    float sm = (os.rmax[m] > -INFINITY) ? os.rsum[m] * expf(os.rmax[m] - mx) : 0.f;
    for (int w = 0; w < NWARP; ++w) {
      const float wm = os.wrmax[w * M + m];
      if (wm > -INFINITY) sm += os.wrsum[w * M + m] * expf(wm - mx);
    }
    os.rmax[m] = mx;
    os.rsum[m] = sm;
    // the token's list in registers: each warp's entries go in with independent comparisons, no chain of
    // dependent shared-memory loads and stores per entry
    float* tv = os.topv + m * KTOP;
    int* ti = os.topi + m * KTOP;
    float v[KTOP];
    int id[KTOP];
#pragma unroll
    for (int e = 0; e < KTOP; ++e) v[e] = tv[e], id[e] = ti[e];
#pragma unroll 1
    for (int i = 0; i < NWARP * KTOP; ++i) {  // entry i % KTOP of warp i / KTOP's list
      const int w = i / KTOP, e = i - w * KTOP;
      list_push(v, id, os.wtopv[((size_t)w * M + m) * KTOP + e], os.wtopi[((size_t)w * M + m) * KTOP + e]);
    }
#pragma unroll
    for (int e = 0; e < KTOP; ++e) tv[e] = v[e], ti[e] = id[e];
  }
  csync();
}

// The cluster kernel. Stages: 0 embedding; 1 + 3 l + (0, 1, 2) = S1, S2, S3 of layer l; 3 L + 1 output;
// beam calls (BEAM): 3 L + 2 select, 3 L + 3 the cache reorder. WIDE:
// one-query attention units of at least 256 positions take steps of 32 positions.
// Only the ring position, the exchange parities and the error flag live in registers across stages; the
// rest of the per-CTA state is rebuilt inside each stage from shared memory and the launch parameters, which
// keeps the register allocation of the stage code free of state it does not use.
template <int NT, int QM, bool BEAM, bool WIDE>
__global__ void __launch_bounds__(BLOCK, 1)
    decoder_cl_kernel(const __grid_constant__ PlanDev pd, const __grid_constant__ CallArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + MAXSLOT;
  uint64_t* xbar = empty + MAXSLOT;  // the exchange barriers of a stage (two) and of its LayerNorm
  int* pre = reinterpret_cast<int*>(smem + pd.off_pre);
  uint8_t* ringdata = smem + pd.off_ring;
  uint8_t* work = smem + pd.off_work;
  const int c = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L = pd.L, n_out = 3 * L + 1, n_stages = n_out + 1 + (BEAM ? 2 : 0);
  int* so = reinterpret_cast<int*>(smem + pd.off_sched);
  int* sb = so + NGEMM + 1;
  int* offs = reinterpret_cast<int*>(smem + pd.off_rows);
  if (threadIdx.x == 0) {
    for (int s = 0; s < pd.nslot; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NWARP);
    }
    mbar_init(&xbar[0], 1);
    mbar_init(&xbar[1], 1);
    mbar_init(&xbar[2], 1);
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
  // every CTA of the cluster has initialised its barriers before any CTA sends to them
  cluster_sync_all();
  unsigned long long* evlog = pd.ts ? pd.ts + (size_t)n_stages * pd.P * 4 + (size_t)c * NEV : nullptr;
  int* nev = reinterpret_cast<int*>(smem + pd.off_pre) + 1033;
  if (threadIdx.x == 0) *nev = pd.ev_from > 0 ? NEV : 0;  // (recording starts at stage ev_from)
  __syncthreads();
  const Ctx cx{so, sb, offs, evlog, nev, reinterpret_cast<float*>(smem + pd.off_pre) + 1040};

  if (warp == NWARP) {  // producer
    if (lane == 0) {
      Frames fr;  // (unused by the output stage's schedule; for_chunks takes one)
      fr.total = 0;
      fr.U = pd.U;
      fr.H = pd.H;
      fr.P = 1;
      fr.pre = pre;
      const Cl cl = cluster_view(pd);
      uint32_t i = 0;
      bool dead = false;
      auto put = [&](const void* src, uint32_t piece, int pieces, uint32_t stride, uint64_t pol) {
        if (dead) return;
        const int s = i % pd.nslot;
        if (!mbar_wait(&empty[s], ((i / pd.nslot) & 1) ^ 1, pd.max_spin)) {
          dead = true;
          atomicExch(pd.err, E_ERR_TIMEOUT);
          return;
        }
        if (i >= (uint32_t)pd.inflight) {
          const uint32_t j = i - pd.inflight;
          if (!mbar_wait(&full[j % pd.nslot], (j / pd.nslot) & 1, pd.max_spin)) {
            dead = true;
            atomicExch(pd.err, E_ERR_TIMEOUT);
            return;
          }
        }
        mbar_arrive_expect_tx(&full[s], piece * (uint32_t)pieces);
        for (int q = 0; q < pieces; ++q)
          bulk_g2s(ringdata + (size_t)s * pd.sstride + (size_t)q * piece,
                   reinterpret_cast<const uint8_t*>(src) + (size_t)q * stride, piece, &full[s], pol);
        ++i;
      };
      const uint64_t first = policy_evict_first(), normal = policy_evict_normal();
      for (int g = 1; g <= n_out && !dead; ++g) {
        if (g == n_out) {  // output stage: the grid kernel's block schedule
          for_chunks(pd, a, fr, cx, 8 * L + 1, c, [&](const void* src, uint32_t bytes) { put(src, bytes, 1, 0u, first); });
        } else {
          const int kind = (g - 1) % 3 + 1, l = (g - 1) / 3;
          cl_chunks(pd, a, cl, pre, offs, kind, l, [&](const void* src, uint32_t piece, int pieces, uint32_t stride, bool keep) {
            put(src, piece, pieces, stride, keep ? normal : first);
          });
        }
      }
      const uint32_t from = i > (uint32_t)pd.nslot ? i - pd.nslot : 0;
      for (uint32_t j = from; j < i; ++j) mbar_wait(&full[j % pd.nslot], (j / pd.nslot) & 1, DEFAULT_SPIN);
    }
    return;
  }

  if (threadIdx.x < pd.M) {  // the output stage's running argmax / log-softmax partials and top-K
    OutState os = carve_out(smem + pd.off_out, pd.M, BEAM);
    os.amax[threadIdx.x] = -INFINITY;
    os.aidx[threadIdx.x] = 0x7fffffff;
    os.rmax[threadIdx.x] = -INFINITY;
    os.rsum[threadIdx.x] = 0.f;
    for (int j = 0; j < KTOP; ++j) {
      os.topv[threadIdx.x * KTOP + j] = -INFINITY;
      os.topi[threadIdx.x * KTOP + j] = 0x7fffffff;
    }
  }
  uint32_t ring_i = 0, ph[3] = {0u, 0u, 0u};
  bool dead = false;
  for (int g = 0; g < n_stages; ++g) {
    unsigned long long* ts = pd.ts ? pd.ts + ((size_t)g * pd.P + c) * 4 : nullptr;
    if (cx.ev && threadIdx.x == 0 && g == pd.ev_from && g > 0) *cx.nev = 0;
    if (ts && threadIdx.x == 0) ts[0] = globaltimer();
    Ring ring{full, empty, ringdata, pd.nslot, pd.sstride, ring_i, pd.max_spin, pd.err, dead, 0ull, pd.ts != nullptr};
    // A failed call (this CTA's or another's timed-out wait, known to every thread of the CTA from the last grid
    // barrier) runs no further stage: no exchange barrier is armed again while one of its phases may still be
    // open, and no exchange is sent. Inside a live stage every sender sends, so each phase armed there completes.
    if (dead) {
    } else if (g == 0) {
      cl_embed(pd, a, cx, c);
    } else if (g < n_out) {
      const int kind = (g - 1) % 3 + 1, l = (g - 1) / 3;
      const long long* xin = pd.xf[(g - 1) % 3];
      long long* xout = pd.xf[g % 3];
      long long* xfree = pd.xf[(g + 1) % 3];
      const Cl cl = cluster_view(pd);
      const int busy = CS * (kind < 3 ? pd.H * pd.RG : pd.NCL3);  // CTAs 0 .. busy - 1 have stage work
      const int gres = kind == 1 ? G_WO : (kind == 2 ? G_WCO : G_F2);
      if (busy < pd.P) {
        if (c >= busy) cl_residual(pd, gres, l, xin, xout, xfree, c - busy, pd.P - busy);
      } else {
        cl_residual(pd, gres, l, xin, xout, xfree, c, pd.P);
      }
      event(cx, 50);
      if (kind < 3) {
        if (cl.cid < pd.H * pd.RG && cl.Mg > 0)
          cl_attn_stage<NT, QM, WIDE>(pd, a, ring, cx, cl, pre, kind, l, work, xbar, ph, xin, xout);
      } else if (cl.ffn) {
        cl_ffn_stage<NT>(pd, ring, cx, cl, work, xbar, ph, xin, xout);
      }
      event(cx, 57);
      // (no per-thread fence: the grid barrier's release by thread 0 after the CTA barrier publishes the
      // stage's writes, as in the grid-stage kernel)
    } else if (g == n_out) {
      OutState os = carve_out(smem + pd.off_out, pd.M, BEAM);
      if (BEAM) {
        cl_out_stage_beam<NT>(pd, a, ring, cx, work, os, &xbar[2], ph[2]);
        beam_partials(pd, c, os);
      } else {
        int* flag = reinterpret_cast<int*>(smem + pd.off_pre) + 1032;
        cl_out_stage<NT>(pd, a, ring, cx, work, os, &xbar[2], ph[2]);
        event(cx, 72);
        if (a.pred) argmax_finish(pd, a, c, os, flag, work);
      }
    } else if (BEAM) {
      if (g == n_out + 1) select_stage(pd, a, cx, c, work);
      else reorder_stage(pd, a, cx, c, work);
    }
    ring_i = ring.i;
    dead = ring.dead;
    if (ts && threadIdx.x == 0) ts[1] = globaltimer();
    if (g < n_stages - 1) grid_sync(pd, (uint32_t)(g + 1) * pd.P, dead, reinterpret_cast<int*>(smem + pd.off_pre) + 1034);
    if (ts && threadIdx.x == 0) {
      ts[2] = globaltimer();
      ts[3] = ring.waited;
    }
  }
  csync();
  if (threadIdx.x == 0) {
    if (atom_acq_rel_add(&pd.ctr[1], 1) == (uint32_t)(pd.P - 1)) {
      atomicExch(&pd.ctr[1], 0u);
      atomicExch(&pd.ctr[0], 0u);
    }
  }
  // no CTA leaves while another CTA of its cluster may still address its shared memory (an exchange store
  // sent late after a timed-out wait); the producer warps, exited, do not count
  cluster_sync_all();
}

}  // namespace owsm
