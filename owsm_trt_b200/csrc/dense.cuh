// The dense kernel: decoder calls of 33 to 64 tokens (rows x window), where the layer GEMMs are dense enough for
// the fifth-generation tensor cores. Included by decoder.cu after cluster.cuh (it uses the ring, the attention
// units of the cluster kernel, the embedding and argmax stages of the grid-stage kernel).
//
// Stages (one grid barrier after each): embedding; per layer QKV (LN1 folded), self-attention, out-projection
// + residual, cross-Q (LN2), cross-attention, cross-out + residual, FFN1 (LN3) + ReLU, FFN2 + residual; the
// vocabulary projection (final LN) with the fused argmax.
//
// GEMMs y[token, n] = sum_k W[n, k] x[token, k] run swap-AB on tcgen05: the weights are the M = 128 operand
// (a tile of 128 output rows), the call's tokens (padded to 64) the N = 64 operand, the fp32 accumulator
// 128 TMEM lanes x 64 columns. A work item is (tile, K range): the weights of the range stream through the
// ring as 16 KB chunks (128 rows x 64 k) prepacked in the canonical K-major layout (core matrices of 8 rows x 8
// k, 128 contiguous bytes; k groups 2 KB apart, row groups 128 bytes apart), so a bulk copy lands them ready for
// the MMA; the token operand (the range of the normalised residual rows, or of the attention / FFN output) sits
// in shared memory in the same layout (k groups 8 x 128 bytes apart). One thread issues the MMAs; a finished
// ring slot is handed back by tcgen05.commit; the item's accumulator is read by warps 0-3 (one TMEM lane
// quarter each: a thread owns one output row and its 64 token columns).
// A tile whose K is split writes each range's partial sums to global memory; the last range to arrive (counted
// per tile) adds them up in range order -- the result does not depend on the arrival order -- and applies the
// epilogue (bias, residual add, ReLU, fp16 stores, logits and argmax).
// Attention: a unit is a (row, head) of self-attention or an (utterance, head) of cross-attention with all of its
// positions, so no unit is split across CTAs; its warps step through the positions in parallel (attn_unit) and the
// normalised output goes to the next GEMM's operand layout in global memory.

#pragma once
#include "tc.cuh"

namespace owsm {

constexpr int DN_MT = 8;                 // token groups of 8: up to 64 tokens
constexpr int DN_TOK = DN_MT * 8;
constexpr int DN_TILE = 128;             // weight rows per tile
constexpr int DN_KR = 512;               // largest operand half (64 tokens x 512 fp16 = 64 KB of shared memory)
constexpr int DN_KI = 1024;              // largest K range of a work item (FFN2 splits its K in ranges of this size)
constexpr int DN_CHUNK = DN_TILE * 64 * 2;  // bytes of a 128 x 64 weight chunk
constexpr int DN_BBYTES = DN_TOK * DN_KR * 2;

// K ranges of a GEMM's work items (at most DN_KI features, a multiple of 128), and the halves an item streams its
// token operand in (at most DN_KR features, a multiple of 128: a half is a whole number of two-chunk ring slots).
__host__ __device__ constexpr int dn_splits(int K) {
  int n = (K + DN_KI - 1) / DN_KI;
  while (K % n || (K / n) % 128) ++n;
  return n;
}
// The GEMMs after a LayerNorm read the residual itself, as fp16 high and low parts (two MMAs per K slice), and
// apply the normalisation in the epilogue: y = rstd (W' x - mean c) + b', c = W' 1 (the reference megakernel's
// algebra, src/owsm_trt/megakernel.py:82-117, :150-250). Their operand parts carry both halves of a K range.
__host__ __device__ constexpr bool dn_hilo(int gi) { return gi == 0 /*QKV*/ || gi == 2 /*CQ*/ || gi == 4 /*F1*/ || gi == 6 /*OUT*/; }
// The parts an item streams its token operand in: at most DN_KR / 2 features with high and low parts (64 KB), at
// most DN_KR otherwise, a multiple of 128 (a whole number of two-chunk ring slots).
__host__ __device__ constexpr int dn_parts(int kr, bool hilo) {
  const int mx = hilo ? DN_KR / 2 : DN_KR;
  int n = (kr + mx - 1) / mx;
  while (kr % n || (kr / n) % 128) ++n;
  return n;
}

// Index (halves) of element (token m, feature k) in the token-operand layout: blocks of 64 features (8 KB: 64
// token rows of 128 bytes), a row's 16-byte chunks XOR-swizzled by the token's row within its group of 8 -- the
// K-major 128-byte-swizzle layout of the tensor cores (8-row groups 1024 bytes apart), so a warp writing one
// token's consecutive 8-feature chunks touches every bank once. Blocks must start 1024-byte aligned.
__device__ __forceinline__ int dn_bidx(int m, int k) {
  return ((k >> 6) << 12) + (m << 6) + ((((k >> 3) & 7) ^ (m & 7)) << 3) + (k & 7);
}

// LayerNorm statistics of the residual rows from the partial sums the residual's producers left (xstat
// [D / 128][64 tokens][sum, sum of squares]: one slot per 128-feature tile): mean and 1 / sqrt(var + eps) per token
// into st[64][2] (shared memory), fp64 over the slots; padding tokens 0.
__device__ __forceinline__ void dn_stats(const PlanDev& pd, float* st) {
  const int m = threadIdx.x;
  if (m < DN_TOK) {
    float mean = 0.f, rs = 0.f;
    if (m < pd.M) {
      double s1 = 0.0, s2 = 0.0;
      for (int sl = 0; sl < (pd.D >> 7); ++sl) {
        const float2 p = __ldcg(reinterpret_cast<const float2*>(pd.xstat) + (size_t)sl * DN_TOK + m);
        s1 += p.x;
        s2 += p.y;
      }
      const double mu = s1 / pd.D, var = fmax(s2 / pd.D - mu * mu, 0.0);
      mean = (float)mu;
      rs = (float)(1.0 / sqrt(var + (double)pd.eps));
    }
    st[2 * m] = mean;
    st[2 * m + 1] = rs;
  }
}

// The token operand of features [k0, k0 + hs) from a global buffer in the same layout (attention output, FFN
// hidden): one bulk copy of the contiguous range, issued and awaited by thread 0 (the MMA issuer).
// With lo (the low parts of the residual operand), a second range of the same features follows in the operand.
__device__ __forceinline__ bool dn_stage_copy(const __half* src, const __half* lo, int k0, int hs, __half* bbuf,
                                              uint64_t* bar, uint32_t& ph, uint32_t spin) {
  // the source was written by other CTAs' ordinary stores before the grid barrier: order them before the
  // bulk-copy engine's reads
  asm volatile("fence.proxy.async.global;" ::: "memory");
  const uint32_t bytes = (uint32_t)hs * DN_TOK * 2;
  mbar_arrive_expect_tx(bar, lo ? 2 * bytes : bytes);
  bulk_g2s_nohint(bbuf, src + (size_t)(k0 >> 6) * (DN_TOK * 64), bytes, bar);
  if (lo) bulk_g2s_nohint(bbuf + (size_t)hs * DN_TOK, lo + (size_t)(k0 >> 6) * (DN_TOK * 64), bytes, bar);
  const bool ok = mbar_wait(bar, ph, spin);
  ph ^= 1u;
  return ok;
}

// Completion of this thread's tcgen05 work, counted on an mbarrier: `issued` commits made (thread 0), `seen`
// phases awaited (every consumer thread).
struct TcBar {
  uint64_t* bar;
  uint32_t issued, seen;
};

__device__ __forceinline__ void tc_wait(const PlanDev& pd, Ring& ring, TcBar& b) {
  if (!ring.dead && !mbar_wait(b.bar, b.seen & 1u, ring.spin)) {
    ring.dead = true;
    atomicExch(pd.err, E_ERR_TIMEOUT);
  }
  ++b.seen;
  tc_fence_after();
}

// One GEMM stage of the dense kernel on this CTA: its work items (tile, K range) in schedule order. An item
// streams its token operand in halves: stage(k, hs) fills the operand with features [k, k + hs) (every consumer
// thread calls it; thread 0 issues the half's MMAs after it), the accumulator collects all halves in TMEM.
// epi(tile, y) finishes a tile from its complete sums y [64 tokens][128 rows] (shared memory; every consumer thread
// calls it). A tile whose K is split (FFN2) writes each range's partial sums to global memory; the last range to
// arrive adds all of them in range order (every thread a share) and finishes the tile.
template <class Stage, class Epi>
__device__ void dn_gemm(const PlanDev& pd, Ring& ring, const Ctx& cx, int gi, uint32_t tmem, TcBar& acc, TcBar& opb,
                        __half* bbuf, int* flag, Stage&& stage, Epi&& epi) {
  const int nb0 = cx.so[gi], nb1 = cx.so[gi + 1];
  if (nb0 == nb1) return;
  const bool hilo = dn_hilo(gi);
  const int K = pd.g[gi].K, ns = pd.nsplit[gi], kr = K / ns, nh = dn_parts(kr, hilo), hs = kr / nh;
  const int hslots = hs >> 7;  // ring slots (two 64-wide chunks each) per half
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = nb0; i < nb1; ++i) {
    const int item = cx.sb[i], tile = item / ns, split = item - tile * ns, k0 = split * kr;
    event(cx, 100);
    for (int h = 0; h < nh; ++h) {
      if (h > 0) tc_wait(pd, ring, opb);  // the previous half's MMAs have read the operand
      stage(k0 + h * hs, hs);
      csync();
      event(cx, 101);
      // (a failed call issues nothing more, so at most the last commit is outstanding when the CTA leaves)
      if (threadIdx.x == 0 && !ring.dead) {
        constexpr uint32_t idesc = idesc_f16_f32(DN_TILE, DN_TOK);
        const uint32_t bb = smem_u32(bbuf);
        for (int j = 0; j < hslots; ++j) {
          const uint32_t idx = ring.i + h * hslots + j;
          const uint32_t sa = smem_u32(ring.wait_at(idx));
          tc_fence_after();
#pragma unroll
          for (int ch = 0; ch < 2; ++ch)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const int kl = (2 * j + ch) * 64 + kk * 16;  // feature offset in the part
              const uint64_t ad = plain_desc(sa + ch * DN_CHUNK + kk * 4096, 2048, 128);
              const uint32_t bo = bb + (uint32_t)(kl >> 6) * (DN_TOK * 128) + (uint32_t)(kl & 63) * 2;
              tc_mma_f16(tmem, ad, sw128_desc(bo), idesc, (h | j | ch | kk) != 0);
              if (hilo) tc_mma_f16(tmem, ad, sw128_desc(bo + (uint32_t)hs * DN_TOK * 2), idesc, 1u);
            }
          // the slot goes back to the producer when these MMAs have read it (one arrival), the other warps'
          // share now
          tc_commit(&ring.empty[idx % ring.ns]);
          mbar_arrive_cnt(&ring.empty[idx % ring.ns], NWARP - 1);
        }
        if (h < nh - 1) {
          tc_commit(opb.bar);
          ++opb.issued;
        } else {
          tc_commit(acc.bar);
          ++acc.issued;
        }
        event(cx, 102);
      }
    }
    tc_wait(pd, ring, acc);
    event(cx, 103);
    ring.i += nh * hslots;
    const int row = warp * 32 + lane;
    float* ysm = reinterpret_cast<float*>(bbuf);  // the tile's sums [token][row] (the operand's MMAs are done)
    // 32 token columns of this thread's accumulator row at a time, straight from the TMEM load's registers
    auto columns_to = [&](int m0, float* dst, int stride) {
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)m0, r);
      tmem_ld_wait();
#pragma unroll
      for (int m = 0; m < 32; ++m) dst[(size_t)m * stride] = __uint_as_float(r[m]);
    };
    bool finish = true;
    if (ns == 1) {
      if (warp < 4)
        for (int m0 = 0; m0 < DN_TOK; m0 += 32) columns_to(m0, ysm + m0 * DN_TILE + row, DN_TILE);
    } else {
      float* pt = pd.part + (size_t)tile * ns * DN_TOK * DN_TILE;  // [range][token][row]
      if (warp < 4)
        for (int m0 = 0; m0 < DN_TOK; m0 += 32) columns_to(m0, pt + ((size_t)split * DN_TOK + m0) * DN_TILE + row, DN_TILE);
      __threadfence();
      csync();
      if (threadIdx.x == 0) *flag = (atomicAdd(&pd.tcnt[tile], 1u) == (uint32_t)(ns - 1));
      csync();
      finish = *flag != 0;
      if (finish) {
        __threadfence();
        // the ranges' sums in range order (every thread a share)
        float4* sum = reinterpret_cast<float4*>(ysm);
        const float4* p4 = reinterpret_cast<const float4*>(pt);
        for (int q = threadIdx.x; q < DN_TOK * DN_TILE / 4; q += NTHR) {
          float4 t = __ldcg(p4 + q);
          for (int s2 = 1; s2 < ns; ++s2) {
            const float4 u = __ldcg(p4 + (size_t)s2 * (DN_TOK * DN_TILE / 4) + q);
            t.x += u.x;
            t.y += u.y;
            t.z += u.z;
            t.w += u.w;
          }
          sum[q] = t;
        }
        if (threadIdx.x == 0) atomicExch(&pd.tcnt[tile], 0u);
      }
    }
    csync();
    if (finish) epi(tile, ysm);
    tc_fence_before();
    csync();  // the next item's first MMA overwrites the accumulator (and its staging the operand)
    event(cx, 104);
  }
}

__device__ __forceinline__ void dn_store_hilo(const PlanDev& pd, int m, int n, const float4& r);

// Embedding into the residual rows (a CTA per token) and their LayerNorm partial sums (slot 0 holds the row's
// sums, the other slots zero).
__device__ __noinline__ void dn_embed(const PlanDev& pd, const CallArgs& a, const Ctx& cx, int c) {
  const int D = pd.D, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* red = cx.red;  // [2 * NWARP]
  for (int m = c; m < pd.M; m += pd.P) {
    const int r = m / pd.S, s = m % pd.S;
    long long t = a.tok[(long long)r * a.tok_stride + s];
    t = t < 0 ? 0 : (t >= pd.V ? pd.V - 1 : t);
    long long pos = (long long)cx.offs[r] + s;
    pos = pos >= pd.max_pos ? pd.max_pos - 1 : pos;
    float s1 = 0.f, s2 = 0.f;
    for (int n = 4 * threadIdx.x; n < D; n += 4 * NTHR) {
      float4 v;
      v.x = __half2float(pd.emb[t * D + n]) * pd.xscale + pd.pe[pos * D + n];
      v.y = __half2float(pd.emb[t * D + n + 1]) * pd.xscale + pd.pe[pos * D + n + 1];
      v.z = __half2float(pd.emb[t * D + n + 2]) * pd.xscale + pd.pe[pos * D + n + 2];
      v.w = __half2float(pd.emb[t * D + n + 3]) * pd.xscale + pd.pe[pos * D + n + 3];
      *reinterpret_cast<float4*>(pd.x + (size_t)m * D + n) = v;
      dn_store_hilo(pd, m, n, v);
      s1 += (v.x + v.y) + (v.z + v.w);
      s2 = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, s2))));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    if (lane == 0) {
      red[2 * warp] = s1;
      red[2 * warp + 1] = s2;
    }
    csync();
    for (int sl = threadIdx.x; sl < (D >> 7); sl += NTHR) {
      float2 v = make_float2(0.f, 0.f);
      if (sl == 0)
        for (int w = 0; w < NWARP; ++w) v.x += red[2 * w], v.y += red[2 * w + 1];
      reinterpret_cast<float2*>(pd.xstat)[(size_t)sl * DN_TOK + m] = v;
    }
    csync();
  }
}

// Normalise a unit's partial states (tab [Q][XPS]: unnormalised output dims, max, sum) into the token operand
// layout of the next GEMM: tok(q) = token of query q, k = h * 64 + dim.
template <class Tok>
__device__ __forceinline__ void dn_emit_unit(const float* tab, int Q, int h, __half* dst, Tok&& tok) {
  for (int idx = threadIdx.x; idx < Q * (DK / 8); idx += NTHR) {
    const int q = idx >> 3, d8 = idx & 7;
    const float l = tab[q * XPS + DK + 1];
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const float* o = tab + q * XPS + d8 * 8;
    uint4 w;
    w.x = pack_half2(o[0] * inv, o[1] * inv);
    w.y = pack_half2(o[2] * inv, o[3] * inv);
    w.z = pack_half2(o[4] * inv, o[5] * inv);
    w.w = pack_half2(o[6] * inv, o[7] * inv);
    *reinterpret_cast<uint4*>(dst + dn_bidx(tok(q), h * DK + d8 * 8)) = w;
  }
}

// Self-attention: unit (row b, head h) for u = c, c + P, ...: the row's S queries over its cached positions
// [0, offset) (ring chunks) and its S new keys / values (causal), which are also written to the cache at
// offset .. offset + S - 1 and to new_kv.
template <int QM, bool WIDE>
__device__ __noinline__ void dn_satt(const PlanDev& pd, const CallArgs& a, Ring& ring, const Ctx& cx, int layer, int c,
                        uint8_t* work) {
  const AttnSmem as = carve_attn(work, pd.Qmax);
  float* tab = reinterpret_cast<float*>(work + ((attn_smem(pd.Qmax) + 15) & ~(size_t)15));
  const int S = pd.S, D = pd.D, H = pd.H;
  for (int u = c; u < pd.R * H; u += pd.P) {
    const int b = u / H, h = u - b * H, off = cx.offs[b];
    csync();  // the previous unit's readers of the staging area are done
    for (int idx = threadIdx.x; idx < S * (DK / 8); idx += NTHR) {
      const int q = idx >> 3, d0 = (idx & 7) * 8;
      const __half* row = pd.qkv + (size_t)(b * S + q) * 3 * D + h * DK + d0;
      const uint4 qv = __ldcg(reinterpret_cast<const uint4*>(row));
      const uint4 kv = __ldcg(reinterpret_cast<const uint4*>(row + D));
      const uint4 vv = __ldcg(reinterpret_cast<const uint4*>(row + 2 * D));
      const __half2* q2 = reinterpret_cast<const __half2*>(&qv);
      const __half2* k2 = reinterpret_cast<const __half2*>(&kv);
      const __half2* v2 = reinterpret_cast<const __half2*>(&vv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 fq = __half22float2(q2[e]), fk = __half22float2(k2[e]), fv = __half22float2(v2[e]);
        const int d = q * DK + d0 + 2 * e;
        as.q[d] = fq.x * 0.125f;
        as.q[d + 1] = fq.y * 0.125f;
        if (QM == 1 && WIDE) {
          as.out[qperm(d0 + 2 * e)] = fq.x * 0.125f;
          as.out[qperm(d0 + 2 * e + 1)] = fq.y * 0.125f;
        }
        as.knew[d] = fk.x;
        as.knew[d + 1] = fk.y;
        as.vnew[d] = fv.x;
        as.vnew[d + 1] = fv.y;
      }
      // (layer strides of the caller's buffers: Rs rows, more than R when the call is a row slice)
      const size_t cs = ((((size_t)layer * pd.Rs + b) * H + h) * pd.C + off + q) * DK + d0;
      *reinterpret_cast<uint4*>(a.kc + cs) = kv;
      *reinterpret_cast<uint4*>(a.vc + cs) = vv;
      *reinterpret_cast<uint4*>(a.new_kv + ((((size_t)(layer * 2) * pd.Rs + b) * H + h) * S + q) * DK + d0) = kv;
      *reinterpret_cast<uint4*>(a.new_kv + ((((size_t)(layer * 2 + 1) * pd.Rs + b) * H + h) * S + q) * DK + d0) = vv;
    }
    attn_unit<QM, WIDE>(as, ring, S, 0, off, pd.apos, S, cx,
                        [&](int q, int c4, const float4& v) { sts128f(&tab[q * XPS + c4 * 4], v); });
    csync();
    dn_emit_unit(tab, S, h, pd.obuf, [&](int q) { return b * S + q; });
  }
}

// Cross-attention: unit (utterance uu, head h) for units c, c + P, ...: the utterance's G rows x S queries over
// its first enc_len frames (ring chunks), one unit per CTA at a time (no unit is split).
template <int QM, bool WIDE>
__device__ __noinline__ void dn_xatt(const PlanDev& pd, Ring& ring, const Ctx& cx, const int* pre, int layer, int c,
                        uint8_t* work) {
  const AttnSmem as = carve_attn(work, pd.Qmax);
  float* tab = reinterpret_cast<float*>(work + ((attn_smem(pd.Qmax) + 15) & ~(size_t)15));
  const int S = pd.S, D = pd.D, H = pd.H, G = pd.G, Q = G * S;
  for (int u = c; u < pd.U * H; u += pd.P) {
    const int uu = u / H, h = u - uu * H, len = pre[uu + 1] - pre[uu];
    csync();
    for (int idx = threadIdx.x; idx < Q * (DK / 8); idx += NTHR) {
      const int q = idx >> 3, d0 = (idx & 7) * 8;
      const uint4 qv = __ldcg(reinterpret_cast<const uint4*>(pd.q2 + (size_t)(uu * Q + q) * D + h * DK + d0));
      const __half2* q2 = reinterpret_cast<const __half2*>(&qv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 fq = __half22float2(q2[e]);
        as.q[q * DK + d0 + 2 * e] = fq.x * 0.125f;
        as.q[q * DK + d0 + 2 * e + 1] = fq.y * 0.125f;
        if (QM == 1 && WIDE) {
          as.out[qperm(d0 + 2 * e)] = fq.x * 0.125f;
          as.out[qperm(d0 + 2 * e + 1)] = fq.y * 0.125f;
        }
      }
    }
    attn_unit<QM, WIDE>(as, ring, Q, 0, len, pd.apos, 0, cx,
                        [&](int q, int c4, const float4& v) { sts128f(&tab[q * XPS + c4 * 4], v); });
    csync();
    dn_emit_unit(tab, Q, h, pd.obuf, [&](int q) { return uu * Q + q; });
  }
}

// The producer's copies of stage g on CTA c, in consumption order: f(src, bytes) per ring slot.
template <class Fn>
__device__ void dn_chunks(const PlanDev& pd, const CallArgs& a, const Ctx& cx, const int* pre, int g, int c, Fn&& f) {
  int layer;
  const Kind k = stage_kind(pd, g, layer);
  const int gi = gemm_of(k);
  if (gi >= 0) {
    const int K = pd.g[gi].K, ns = pd.nsplit[gi], nchunk = (K / ns) >> 6, cpt = K >> 6;
    const __half* base = pd.gt[gi] + (k == K_OUT ? 0 : (long long)layer * pd.gtl[gi]);
    for (int i = cx.so[gi]; i < cx.so[gi + 1]; ++i) {
      const int item = cx.sb[i], tile = item / ns, split = item - tile * ns;
      const __half* src = base + ((long long)tile * cpt + (long long)split * nchunk) * (DN_CHUNK / 2);
      for (int j = 0; j < nchunk; j += 2)
        f(src + (long long)j * (DN_CHUNK / 2), (uint32_t)((nchunk - j < 2 ? nchunk - j : 2) * DN_CHUNK));
    }
    return;
  }
  if ((k == K_SATT || k == K_XATT) && pd.Qmax == 1) return;  // one-query units read their positions directly
  if (k == K_SATT) {
    for (int u = c; u < pd.R * pd.H; u += pd.P) {
      const int b = u / pd.H, h = u % pd.H, off = cx.offs[b];
      const long long base = ((((long long)layer * pd.Rs + b) * pd.H + h) * pd.C) * DK;
      for (int j0 = 0; j0 < off; j0 += pd.apos) {
        const int n = off - j0 < pd.apos ? off - j0 : pd.apos;
        f((const void*)(a.kc + base + (long long)j0 * DK), (uint32_t)n * DK * 2);
        f((const void*)(a.vc + base + (long long)j0 * DK), (uint32_t)n * DK * 2);
      }
    }
    return;
  }
  if (k == K_XATT) {
    for (int u = c; u < pd.U * pd.H; u += pd.P) {
      const int uu = u / pd.H, h = u % pd.H, len = pre[uu + 1] - pre[uu];
      const long long base = ((((long long)layer * pd.Us + uu) * pd.H + h) * pd.T) * DK;
      for (int j0 = 0; j0 < len; j0 += pd.apos) {
        const int n = len - j0 < pd.apos ? len - j0 : pd.apos;
        f((const void*)(a.ck + base + (long long)j0 * DK), (uint32_t)n * DK * 2);
        f((const void*)(a.cv + base + (long long)j0 * DK), (uint32_t)n * DK * 2);
      }
    }
  }
}

// One-query attention units (greedy calls: a row's single token, an utterance's single row), a warp per unit with
// no CTA barrier: the warp walks the unit's positions 32 at a time straight from global memory (lane j scores
// position p0 + j against the query held in every lane, in the log2 domain; the warp max and the lanes' running
// sums give the online softmax; the value rows are accumulated two dims per lane, each position's probability
// broadcast from its lane). Self-attention adds the row's new key / value (also written to the cache slot at the
// row's offset and to new_kv). Units are spread over all warps of the grid: unit u on warp u mod (P x 7).
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __noinline__ void dn_attn_q1(const PlanDev& pd, const CallArgs& a, const Ctx& cx, const int* pre, int layer,
                                        int c, bool self) {
  // lane = 8 grp + e: lane group grp takes keys p0 + 4 i + grp (i = 0 .. 7) of each 32-key chunk, lane e of the
  // group holds dims 8 e .. 8 e + 7 of q, of those keys and of the group's output; a key's score is summed over
  // its 8 lanes. Each group keeps its own online-softmax state (max, sum, output), merged over the 4 groups at
  // the end. Loads are uint4 per lane, 512 contiguous bytes per warp instruction; the next chunk's keys and values
  // are loaded while the current chunk is scored.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, grp = lane >> 3, e = lane & 7, H = pd.H, D = pd.D;
  const int nunits = (self ? pd.R : pd.U) * H;
  const float qs = 0.125f * kLog2e;  // 1 / sqrt(64), scores in the log2 domain
  for (int u = c * NWARP + warp; u < nunits; u += pd.P * NWARP) {
    const int r = u / H, h = u - r * H;
    int n;
    const __half *K, *V, *qrow;
    if (self) {
      n = cx.offs[r];
      qrow = pd.qkv + (size_t)r * 3 * D + h * DK;
      const size_t base = (((size_t)layer * pd.Rs + r) * H + h) * pd.C * DK;
      K = a.kc + base;
      V = a.vc + base;
    } else {
      n = pre[r + 1] - pre[r];
      qrow = pd.q2 + (size_t)r * D + h * DK;
      const size_t base = (((size_t)layer * pd.Us + r) * H + h) * pd.T * DK;
      K = a.ck + base;
      V = a.cv + base;
    }
    float q[8];
    {
      const uint4 w = __ldcg(reinterpret_cast<const uint4*>(qrow) + e);
      const __half2* h2 = reinterpret_cast<const __half2*>(&w);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 f = __half22float2(h2[t]);
        q[2 * t] = f.x * qs;
        q[2 * t + 1] = f.y * qs;
      }
    }
    const uint4* K4 = reinterpret_cast<const uint4*>(K) + e;  // key j, this lane's dims: K4[j * 8]
    const uint4* V4 = reinterpret_cast<const uint4*>(V) + e;
    float m = -INFINITY, l = 0.f, o[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) o[t] = 0.f;
    uint4 kc[8], vc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int j = 4 * i + grp;
      kc[i] = j < n ? __ldg(K4 + (size_t)j * 8) : make_uint4(0u, 0u, 0u, 0u);
      vc[i] = j < n ? __ldg(V4 + (size_t)j * 8) : make_uint4(0u, 0u, 0u, 0u);
    }
    for (int p0 = 0; p0 < n; p0 += 32) {
      uint4 kn[8], vn[8];
      const int p1 = p0 + 32;
#pragma unroll
      for (int i = 0; i < 8; ++i) {  // the next chunk, in flight while this one is scored
        const int j = p1 + 4 * i + grp;
        kn[i] = j < n ? __ldg(K4 + (size_t)j * 8) : make_uint4(0u, 0u, 0u, 0u);
        vn[i] = j < n ? __ldg(V4 + (size_t)j * 8) : make_uint4(0u, 0u, 0u, 0u);
      }
      float sc[8], cmax = -INFINITY;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const __half2* h2 = reinterpret_cast<const __half2*>(&kc[i]);
        float acc = 0.f;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float2 f = __half22float2(h2[t]);
          acc = fmaf(f.x, q[2 * t], fmaf(f.y, q[2 * t + 1], acc));
        }
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        acc += __shfl_xor_sync(0xffffffffu, acc, 2);
        acc += __shfl_xor_sync(0xffffffffu, acc, 4);
        sc[i] = p0 + 4 * i + grp < n ? acc : -INFINITY;
        cmax = fmaxf(cmax, sc[i]);
      }
      if (cmax != -INFINITY) {  // (a group with no key left in this chunk keeps its state)
        const float mn = fmaxf(m, cmax);
        const float alpha = exp2f(m - mn);  // 0 while m = -inf
        l *= alpha;
#pragma unroll
        for (int t = 0; t < 8; ++t) o[t] *= alpha;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float pi = exp2f(sc[i] - mn);
          l += pi;
          const __half2* h2 = reinterpret_cast<const __half2*>(&vc[i]);
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const float2 f = __half22float2(h2[t]);
            o[2 * t] = fmaf(pi, f.x, o[2 * t]);
            o[2 * t + 1] = fmaf(pi, f.y, o[2 * t + 1]);
          }
        }
        m = mn;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        kc[i] = kn[i];
        vc[i] = vn[i];
      }
    }
    if (self) {  // the new key / value (causal: the query sees its own position), in group 0's state
      const uint4 kw = __ldcg(reinterpret_cast<const uint4*>(qrow + D) + e);
      const uint4 vw = __ldcg(reinterpret_cast<const uint4*>(qrow + 2 * D) + e);
      const __half2* k2 = reinterpret_cast<const __half2*>(&kw);
      float acc = 0.f;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 f = __half22float2(k2[t]);
        acc = fmaf(f.x, q[2 * t], fmaf(f.y, q[2 * t + 1], acc));
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      acc += __shfl_xor_sync(0xffffffffu, acc, 4);
      if (grp == 0) {
        const float mn = fmaxf(m, acc);
        const float alpha = exp2f(m - mn), pi = exp2f(acc - mn);
        const __half2* v2 = reinterpret_cast<const __half2*>(&vw);
        l = l * alpha + pi;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float2 f = __half22float2(v2[t]);
          o[2 * t] = fmaf(pi, f.x, o[2 * t] * alpha);
          o[2 * t + 1] = fmaf(pi, f.y, o[2 * t + 1] * alpha);
        }
        m = mn;
        const size_t cs = ((((size_t)layer * pd.Rs + r) * H + h) * pd.C + n) * DK;
        reinterpret_cast<uint4*>(a.kc + cs)[e] = kw;
        reinterpret_cast<uint4*>(a.vc + cs)[e] = vw;
        reinterpret_cast<uint4*>(a.new_kv + ((((size_t)(layer * 2) * pd.Rs + r) * H + h)) * DK)[e] = kw;
        reinterpret_cast<uint4*>(a.new_kv + ((((size_t)(layer * 2 + 1) * pd.Rs + r) * H + h)) * DK)[e] = vw;
      }
    }
#pragma unroll
    for (int off = 8; off <= 16; off <<= 1) {  // merge the groups' states
      const float mo = __shfl_xor_sync(0xffffffffu, m, off), lo = __shfl_xor_sync(0xffffffffu, l, off);
      const float mn = fmaxf(m, mo);
      const float a1 = m == -INFINITY ? 0.f : exp2f(m - mn), a2 = mo == -INFINITY ? 0.f : exp2f(mo - mn);
      l = l * a1 + lo * a2;
#pragma unroll
      for (int t = 0; t < 8; ++t) o[t] = o[t] * a1 + __shfl_xor_sync(0xffffffffu, o[t], off) * a2;
      m = mn;
    }
    if (grp == 0) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint4 w;
      w.x = pack_half2(o[0] * inv, o[1] * inv);
      w.y = pack_half2(o[2] * inv, o[3] * inv);
      w.z = pack_half2(o[4] * inv, o[5] * inv);
      w.w = pack_half2(o[6] * inv, o[7] * inv);
      *reinterpret_cast<uint4*>(pd.obuf + dn_bidx(r, h * DK + 8 * e)) = w;
    }
  }
}

// ---- tile epilogues: every consumer thread, item idx = (token m, rows 4 g .. 4 g + 3) of a tile's sums
// y [64 tokens][128 rows] (shared memory), a warp per token (its 32 lanes cover the 128 rows); out of line (once
// per tile), so the stage loops keep their registers.

// Four residual values of token m (features n .. n + 3) into the GEMM operand as fp16 high and low parts.
__device__ __forceinline__ void dn_store_hilo(const PlanDev& pd, int m, int n, const float4& r) {
  const __half2 h0 = __floats2half2_rn(r.x, r.y), h1 = __floats2half2_rn(r.z, r.w);
  const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
  uint2 hi, lo;
  hi.x = *reinterpret_cast<const uint32_t*>(&h0);
  hi.y = *reinterpret_cast<const uint32_t*>(&h1);
  lo.x = pack_half2(r.x - f0.x, r.y - f0.y);
  lo.y = pack_half2(r.z - f1.x, r.w - f1.y);
  const int i = dn_bidx(m, n);
  *reinterpret_cast<uint2*>(pd.xop + i) = hi;
  *reinterpret_cast<uint2*>(pd.xop + (size_t)pd.D * DN_TOK + i) = lo;
}

// residual: x[m][n] += y + b, its fp16 high / low operand parts, and the LayerNorm partial sums of the tile's 128
// features per token
__device__ __noinline__ void dn_epi_res(const PlanDev& pd, const float* y, const float* bias, int tile) {
  constexpr int B = 4;
  const int D = pd.D, n_items = pd.M * 32;
  for (int base = threadIdx.x; base < n_items; base += B * NTHR) {
    float4 xo[B];
#pragma unroll
    for (int j = 0; j < B; ++j) {
      const int idx = base + j * NTHR;
      if (idx < n_items) xo[j] = __ldcg(reinterpret_cast<const float4*>(pd.x + (size_t)(idx >> 5) * D + tile * DN_TILE) + (idx & 31));
    }
#pragma unroll
    for (int j = 0; j < B; ++j) {
      const int idx = base + j * NTHR, m = idx >> 5, g = idx & 31;
      if (idx >= n_items) break;  // (warp-uniform: n_items is a multiple of 32)
      const float4 v = reinterpret_cast<const float4*>(y)[m * (DN_TILE / 4) + g];
      const float4 b = __ldg(reinterpret_cast<const float4*>(bias + tile * DN_TILE) + g);
      const float4 r = make_float4(xo[j].x + v.x + b.x, xo[j].y + v.y + b.y, xo[j].z + v.z + b.z, xo[j].w + v.w + b.w);
      reinterpret_cast<float4*>(pd.x + (size_t)m * D + tile * DN_TILE)[g] = r;
      dn_store_hilo(pd, m, tile * DN_TILE + 4 * g, r);
      float s1 = (r.x + r.y) + (r.z + r.w);
      float s2 = fmaf(r.x, r.x, fmaf(r.y, r.y, fmaf(r.z, r.z, r.w * r.w)));
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        s1 += __shfl_xor_sync(0xffffffffu, s1, o);
        s2 += __shfl_xor_sync(0xffffffffu, s2, o);
      }
      if ((threadIdx.x & 31) == 0) reinterpret_cast<float2*>(pd.xstat)[(size_t)tile * DN_TOK + m] = make_float2(s1, s2);
    }
  }
}

// The LayerNorm applied to a GEMM of the raw residual: rstd (acc - mean c) for 4 rows of token m (st [64][mean,
// rstd] in shared memory, c the weights' row sums).
__device__ __forceinline__ float4 dn_norm(const float4& acc, const float* st, const float* cs, int m, int n) {
  const float mu = st[2 * m], rs = st[2 * m + 1];
  const float4 c = __ldg(reinterpret_cast<const float4*>(cs + n));
  return make_float4(rs * (acc.x - mu * c.x), rs * (acc.y - mu * c.y), rs * (acc.z - mu * c.z), rs * (acc.w - mu * c.w));
}

// fp16 outputs out[m][ld] (q / k / v, cross queries): LN-corrected y + b
__device__ __noinline__ void dn_epi_half(const PlanDev& pd, const float* y, const float* bias, const float* st,
                                         const float* cs, int tile, __half* out, int ld) {
  for (int idx = threadIdx.x; idx < pd.M * 32; idx += NTHR) {
    const int m = idx >> 5, g = idx & 31;
    const float4 v = dn_norm(reinterpret_cast<const float4*>(y)[m * (DN_TILE / 4) + g], st, cs, m, tile * DN_TILE + 4 * g);
    const float4 b = __ldg(reinterpret_cast<const float4*>(bias + tile * DN_TILE) + g);
    uint2 h;
    h.x = pack_half2(v.x + b.x, v.y + b.y);
    h.y = pack_half2(v.z + b.z, v.w + b.w);
    *reinterpret_cast<uint2*>(out + (size_t)m * ld + tile * DN_TILE + 4 * g) = h;
  }
}

// ReLU(LN-corrected y + b) into the FFN2 operand layout; padding tokens zero
__device__ __noinline__ void dn_epi_relu(const PlanDev& pd, const float* y, const float* bias, const float* st,
                                         const float* cs, int tile) {
  for (int idx = threadIdx.x; idx < DN_TOK * 32; idx += NTHR) {
    const int m = idx >> 5, g = idx & 31;
    uint2 h = make_uint2(0u, 0u);
    if (m < pd.M) {
      const float4 v = dn_norm(reinterpret_cast<const float4*>(y)[m * (DN_TILE / 4) + g], st, cs, m, tile * DN_TILE + 4 * g);
      const float4 b = __ldg(reinterpret_cast<const float4*>(bias + tile * DN_TILE) + g);
      h.x = pack_half2(fmaxf(v.x + b.x, 0.f), fmaxf(v.y + b.y, 0.f));
      h.y = pack_half2(fmaxf(v.z + b.z, 0.f), fmaxf(v.w + b.w, 0.f));
    }
    *reinterpret_cast<uint2*>(pd.hbuf + dn_bidx(m, tile * DN_TILE + 4 * g)) = h;
  }
}

// logits = y + b, and each warp's running best per token (first index on ties; ids first_time .. last_time left
// out for the rows flagged <notimestamps>)
__device__ __noinline__ void dn_epi_out(const PlanDev& pd, const CallArgs& a, const float* y, const float* bias,
                                        const float* st, const float* cs, int tile, OutState& os) {
  const int M = pd.M, V = pd.V, w = threadIdx.x >> 5;
  for (int idx = threadIdx.x; idx < M * 32; idx += NTHR) {
    const int m = idx >> 5, g = idx & 31;
    const float4 v = dn_norm(reinterpret_cast<const float4*>(y)[m * (DN_TILE / 4) + g], st, cs, m, tile * DN_TILE + 4 * g);
    const float vv[4] = {v.x, v.y, v.z, v.w};
    const int n0 = tile * DN_TILE + 4 * g;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int n = n0 + e;
      if (n < V) {
        const float yv = vv[e] + bias[n];
        a.logits[(size_t)m * V + n] = yv;
        if (!argmax_bad(pd, a, os.topi + m * KTOP, m, n)) merge_best(bv, bi, yv, n);
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      merge_best(bv, bi, ov, oi);
    }
    if ((threadIdx.x & 31) == 0) merge_best(os.wamax[w * M + m], os.waidx[w * M + m], bv, bi);
  }
}

template <int QM, bool WIDE>
__global__ void __launch_bounds__(BLOCK, 1)
    decoder_dense_kernel(const __grid_constant__ PlanDev pd, const __grid_constant__ CallArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + MAXSLOT;
  uint64_t* accbar = empty + MAXSLOT;  // the accumulator of an item is complete
  uint64_t* opbar = accbar + 1;        // an operand half has been read by its MMAs
  uint64_t* bbar = opbar + 1;          // an operand copy has landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bbar + 1);
  int* pre = reinterpret_cast<int*>(smem + pd.off_pre);
  uint8_t* ringdata = smem + pd.off_ring;
  uint8_t* work = smem + pd.off_work;
  __half* bbuf = reinterpret_cast<__half*>(work);
  const int c = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_stages = 8 * pd.L + 2;
  int* so = reinterpret_cast<int*>(smem + pd.off_sched);
  int* sb = so + NGEMM + 1;
  int* offs = reinterpret_cast<int*>(smem + pd.off_rows);
  if (threadIdx.x == 0) {
    for (int s = 0; s < pd.nslot; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NWARP);
    }
    mbar_init(accbar, 1);
    mbar_init(opbar, 1);
    mbar_init(bbar, 1);
    fence_barrier_init();
    pre[0] = 0;
    for (int u = 0; u < pd.U; ++u) pre[u + 1] = pre[u] + utt_len(pd, a, u);
    so[0] = 0;
    for (int gi = 0; gi < NGEMM; ++gi) so[gi + 1] = so[gi] + (pd.goff[gi][c + 1] - pd.goff[gi][c]);
  }
  if (warp == 0) {  // the accumulator: 128 lanes x 64 columns of this SM's tensor memory
    tmem_alloc(tmem_slot, DN_TOK);
    tmem_relinquish();
  }
  for (int r = threadIdx.x; r < pd.R; r += BLOCK) offs[r] = row_off_global(pd, a, r);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  for (int gi = 0; gi < NGEMM; ++gi) {
    const int base = pd.goff[gi][c];
    for (int i = threadIdx.x; i < so[gi + 1] - so[gi]; i += BLOCK) sb[so[gi] + i] = pd.gblk[gi][base + i];
  }
  __syncthreads();
  unsigned long long* evlog = pd.ts ? pd.ts + (size_t)n_stages * pd.P * 4 + (size_t)c * NEV : nullptr;
  int* nev = reinterpret_cast<int*>(smem + pd.off_pre) + 1033;
  if (threadIdx.x == 0) *nev = pd.ev_from > 0 ? NEV : 0;  // (recording starts at stage ev_from)
  __syncthreads();
  const Ctx cx{so, sb, offs, evlog, nev, reinterpret_cast<float*>(smem + pd.off_pre) + 1040};

  if (warp == NWARP) {  // producer: the CTA's whole sequence of copies, as in the grid-stage kernel
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      uint32_t i = 0;
      bool dead = false;
      for (int g = 0; g < n_stages && !dead; ++g) {
        dn_chunks(pd, a, cx, pre, g, c, [&](const void* src, uint32_t bytes) {
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
          mbar_arrive_expect_tx(&full[s], bytes);
          bulk_g2s(ringdata + (size_t)s * pd.sstride, src, bytes, &full[s], pol);
          ++i;
        });
      }
      const uint32_t first = i > (uint32_t)pd.nslot ? i - pd.nslot : 0;
      for (uint32_t j = first; j < i; ++j) mbar_wait(&full[j % pd.nslot], (j / pd.nslot) & 1, DEFAULT_SPIN);
    }
    return;
  }

  Ring ring{full, empty, ringdata, pd.nslot, pd.sstride, 0, pd.max_spin, pd.err, false, 0ull, pd.ts != nullptr};
  bool dead = false;
  if ((smem_u32(bbuf) & 1023u) != 0) {  // the swizzled operand needs 1024-byte alignment: refuse rather than misread
    if (threadIdx.x == 0) atomicExch(pd.err, E_ERR_TIMEOUT);
    dead = true;
  }
  OutState os = carve_out(smem + pd.off_out, pd.M, false);
  for (int m = threadIdx.x; m < pd.M; m += NTHR) {
    os.amax[m] = -INFINITY;
    os.aidx[m] = 0x7fffffff;
  }
  int* flag = reinterpret_cast<int*>(smem + pd.off_pre) + 1032;
  int* tflag = reinterpret_cast<int*>(smem + pd.off_pre) + 1035;
  float* st = reinterpret_cast<float*>(smem + pd.off_stat);  // [64][mean, rstd] of the stage's LayerNorm
  TcBar acc{accbar, 0, 0}, opb{opbar, 0, 0};
  uint32_t bph = 0;
  bool copies = false;  // thread 0: an operand copy was issued (its completion is awaited before the CTA exits)
  const int D = pd.D, M = pd.M, V = pd.V;
  for (int g = 0; g < n_stages; ++g) {
    int layer;
    const Kind k = stage_kind(pd, g, layer);
    unsigned long long* ts = pd.ts ? pd.ts + ((size_t)g * pd.P + c) * 4 : nullptr;
    if (cx.ev && threadIdx.x == 0 && g == pd.ev_from && g > 0) *cx.nev = 0;
    if (ts && threadIdx.x == 0) ts[0] = globaltimer();
    ring.dead = dead;
    const int gi = gemm_of(k);
    const int N = gi >= 0 ? pd.g[gi].N : 0;
    const float* bias = gi >= 0 ? pd.g[gi].b + (k == K_OUT ? 0 : (long long)layer * N) : nullptr;
    auto copy_stage = [&](const __half* src, const __half* lo) {
      return [&, src, lo](int k0, int hs) {
        if (threadIdx.x == 0 && !ring.dead) {
          copies = true;
          if (!dn_stage_copy(src, lo, k0, hs, bbuf, bbar, bph, ring.spin)) {
            ring.dead = true;
            atomicExch(pd.err, E_ERR_TIMEOUT);
          }
        }
      };
    };
    auto res_epi = [&](int tile, const float* y) { dn_epi_res(pd, y, bias, tile); };
    const float* cs = gi >= 0 && pd.gcs[gi] ? pd.gcs[gi] + (k == K_OUT ? 0 : (long long)layer * N) : nullptr;
    auto half_epi = [&](__half* out, int ld) {
      return [&, out, ld](int tile, const float* y) { dn_epi_half(pd, y, bias, st, cs, tile, out, ld); };
    };
    const auto ln_stage = copy_stage(pd.xop, pd.xop + (size_t)D * DN_TOK);
    if (k == K_QKV || k == K_CQ || k == K_F1 || k == K_OUT) {
      if (!dead && cx.so[gi] < cx.so[gi + 1]) {
        dn_stats(pd, st);
        csync();
      }
    }
    if (dead) {
    } else if (k == K_EMBED) {
      dn_embed(pd, a, cx, c);
    } else if (k == K_QKV) {
      dn_gemm(pd, ring, cx, G_QKV, tmem, acc, opb, bbuf, tflag, ln_stage, half_epi(pd.qkv, 3 * D));
    } else if (k == K_SATT) {
      if (QM == 1) dn_attn_q1(pd, a, cx, pre, layer, c, true);
      else dn_satt<QM, WIDE>(pd, a, ring, cx, layer, c, work);
    } else if (k == K_WO || k == K_WCO) {
      dn_gemm(pd, ring, cx, gi, tmem, acc, opb, bbuf, tflag, copy_stage(pd.obuf, nullptr), res_epi);
    } else if (k == K_CQ) {
      dn_gemm(pd, ring, cx, G_CQ, tmem, acc, opb, bbuf, tflag, ln_stage, half_epi(pd.q2, D));
    } else if (k == K_XATT) {
      if (QM == 1) dn_attn_q1(pd, a, cx, pre, layer, c, false);
      else dn_xatt<QM, WIDE>(pd, ring, cx, pre, layer, c, work);
    } else if (k == K_F1) {
      dn_gemm(pd, ring, cx, G_F1, tmem, acc, opb, bbuf, tflag, ln_stage,
              [&](int tile, const float* y) { dn_epi_relu(pd, y, bias, st, cs, tile); });
    } else if (k == K_F2) {
      dn_gemm(pd, ring, cx, G_F2, tmem, acc, opb, bbuf, tflag, copy_stage(pd.hbuf, nullptr), res_epi);
    } else if (k == K_OUT) {
      for (int m = lane; m < M; m += 32) {  // this warp's running best per token
        os.wamax[warp * M + m] = -INFINITY;
        os.waidx[warp * M + m] = 0x7fffffff;
      }
      if (a.rules)  // the timestamp-rule state of every token (dn_gemm's operand staging syncs before its epilogues)
        for (int m = threadIdx.x; m < M; m += NTHR) rule_state(pd, a, m, os.topi + m * KTOP);
      __syncwarp();
      dn_gemm(pd, ring, cx, G_OUT, tmem, acc, opb, bbuf, tflag, ln_stage,
              [&](int tile, const float* y) { dn_epi_out(pd, a, y, bias, st, cs, tile, os); });
      csync();
      for (int m = threadIdx.x; m < M; m += NTHR) {
        float bv = os.amax[m];
        int bi = os.aidx[m];
        for (int w = 0; w < NWARP; ++w) merge_best(bv, bi, os.wamax[w * M + m], os.waidx[w * M + m]);
        os.amax[m] = bv;
        os.aidx[m] = bi;
      }
      csync();
      if (a.pred) argmax_finish(pd, a, c, os, flag, work);
    }
    // the operands just written (residual parts, attention output, FFN hidden) are read by a later stage's bulk
    // copies (async proxy)
    if (k != K_QKV && k != K_CQ && k != K_OUT) asm volatile("fence.proxy.async.global;" ::: "memory");
    dead = dead || ring.dead;
    if (ts && threadIdx.x == 0) ts[1] = globaltimer();
    if (g < n_stages - 1) grid_sync(pd, (uint32_t)(g + 1) * pd.P, dead, reinterpret_cast<int*>(smem + pd.off_pre) + 1034);
    if (ts && threadIdx.x == 0) {
      ts[2] = globaltimer();
      ts[3] = ring.waited;
    }
    ring.waited = 0;
  }
  csync();
  if (threadIdx.x == 0) {
    if (atom_acq_rel_add(&pd.ctr[1], 1) == (uint32_t)(pd.P - 1)) {
      atomicExch(&pd.ctr[1], 0u);
      atomicExch(&pd.ctr[0], 0u);
    }
  }
  // before the CTA leaves: its last MMAs and operand copy (which a timed-out wait may have left running) are
  // done -- both always finish, so the default limit -- then the accumulator columns are freed
  if (threadIdx.x == 0) {
    if (acc.issued) mbar_wait(accbar, (acc.issued - 1) & 1u, DEFAULT_SPIN);
    if (opb.issued) mbar_wait(opbar, (opb.issued - 1) & 1u, DEFAULT_SPIN);
    if (copies) mbar_wait(bbar, bph ^ 1u, DEFAULT_SPIN);
  }
  tc_fence_before();
  csync();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, DN_TOK);
  }
}

// Fragment-ordered weights (the mma.sync packing of owsm_dec_create) -> 128-row tiles for the dense kernel:
// out[layer][tile][K / 64][k group 8][row group 16][row 8][8 k] (halves; rows >= N zero; out_lstride halves per
// layer). A thread writes one 16-byte core-matrix row from four 32-bit fragment registers.
__global__ void tile_pack_kernel(const uint4* __restrict__ frag, int N, int K, int bstride, long long lstride,
                                 int layers, __half* __restrict__ out, long long out_lstride) {
  const int ntile = (N + DN_TILE - 1) / DN_TILE, nchunk = K >> 6;
  const long long per_layer = (long long)ntile * nchunk * 8 * 16 * 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < per_layer * layers;
       i += (long long)gridDim.x * blockDim.x) {
    const int layer = (int)(i / per_layer);
    long long j = i - (long long)layer * per_layer;
    const int r = (int)(j & 7);
    j >>= 3;
    const int rg = (int)(j & 15);
    j >>= 4;
    const int kg = (int)(j & 7);
    j >>= 3;
    const int chunk = (int)(j % nchunk), tile = (int)(j / nchunk);
    const int row = tile * DN_TILE + rg * 8 + r, k0 = chunk * 64 + kg * 8;
    uint4 o = make_uint4(0u, 0u, 0u, 0u);
    if (row < N) {
      // fragment order: block row >> 4, k block k0 >> 4; lane g * 4 + t holds rows g, g + 8 x k 2t, 2t + 1 (regs 0,
      // 1) and k 2t + 8, 2t + 9 (regs 2, 3)
      const int rb = row >> 4, rr = row & 15, g = rr & 7, hi = rr >> 3, kb = k0 >> 4, khi = (k0 & 15) >> 3;
      const uint4* src = frag + (long long)layer * lstride + (long long)rb * bstride + kb * 32 + g * 4;
      uint32_t w[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const uint4 f = src[t];
        const uint32_t regs[4] = {f.x, f.y, f.z, f.w};
        w[t] = regs[hi + 2 * khi];
      }
      o = make_uint4(w[0], w[1], w[2], w[3]);
    }
    // (16-byte units: out_lstride counts halves)
    const long long dst = (long long)layer * (out_lstride >> 3) + ((((long long)tile * nchunk + chunk) * 8 + kg) * 16 + rg) * 8 + r;
    reinterpret_cast<uint4*>(out)[dst] = o;
  }
}

// Row sums of the tile-packed fp16 weights (fp32 sums of the fp16 values): cs[layer][n], n < N.
__global__ void tile_rowsum_kernel(const __half* __restrict__ t, int N, int K, int layers, long long lstride,
                                   float* __restrict__ cs) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N * layers) return;
  const int layer = i / N, row = i - layer * N, tile = row / DN_TILE, rg = (row % DN_TILE) >> 3, r = row & 7;
  const int nchunk = K >> 6;
  float s = 0.f;
  for (int ch = 0; ch < nchunk; ++ch)
    for (int kg = 0; kg < 8; ++kg) {
      const __half* p = t + (long long)layer * lstride + ((((long long)tile * nchunk + ch) * 8 + kg) * 16 + rg) * 64 + r * 8;
#pragma unroll
      for (int e = 0; e < 8; ++e) s += __half2float(p[e]);
    }
  cs[i] = s;
}

}  // namespace owsm
