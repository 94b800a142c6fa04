// dense_maxsim.cu -- fused MaxSim on the sm_100a tensor cores.
//
//   score[q, doc] = sum_i max_{j in doc} <Q[q,i,:], D[j,:]>
//
// Reference semantics: src/flash_maxsim_v2.py:73-130 (_flash_maxsim_v2_multiquery_kernel: query
// block x doc tile dot, row max, running max, sum of the per-token maxima, query rows past Nq add
// 0, doc rows past Nd are masked) and :133-190 (d > 128 accumulates partial dots over d before the
// max); src/flash_maxsim_kernel.py:25-164 (V1: per-query-token maxima, running max starts at -inf
// so an empty document gives -inf) and :248-273 (ragged documents through an offsets array).
//
// B200 design (not a translation of the Triton kernels):
//  * Queries are packed into 128-row "M tiles": every query owns ceil(Nq/32) groups of 32 rows
//    ("chunks"), so one warp's TMEM lane quarter holds exactly one query chunk. The MMA computes
//    S = Qtile . Dtile^T with the query rows on TMEM lanes and doc tokens on TMEM columns.
//  * Doc tokens are streamed as TN-token tiles (TN = 256; 128 in the PQ variant) by TMA (128-byte swizzle) into a
//    ring of shared-memory stages; each D byte is read from HBM once per CTA group.
//  * One thread issues tcgen05.mma (kind::f16 for fp16/bf16, kind::tf32 for fp32 inputs) into a
//    ring of fp32 accumulators in TMEM (512 / TN slots of TN columns).
//  * Epilogue warps read their 32 lanes with tcgen05.ld and run a segmented max along the columns
//    (doc boundaries are warp-uniform, taken from the offsets array), then one warp-shuffle sum over
//    the 32 query-token lanes per finished document. The Nq x Nd similarity matrix never leaves the
//    SM. Rows mode (several query tiles): two groups of four warps take alternate query tiles.
//    Column-split mode (one query tile): the chunks are replicated over the lane quarters and all
//    eight warps share each tile's columns, chaining partial maxima through shared memory.
//  * The epilogue reads every fp32 similarity once from TMEM, and tcgen05.ld sustains ~56 B/clk per
//    SM: for large query batches that, not the tensor pipe, bounds the kernel.
//  * The CTA grid is (token range) x (query group). Token ranges are cut at document boundaries
//    (warp-cooperative binary search on the offsets), so no document straddles two CTAs and no
//    cross-CTA merge or atomic is needed: results are deterministic.
//  * Q-resident mode keeps the CTA's G query tiles in shared memory for the whole range; streaming
//    mode (large d) loads one (query chunk, doc chunk) pair per pipeline stage.
//
// Warp roles (320 threads): warp 0 = TMA producer, warp 1 = TMEM owner + MMA issuer,
// warps 2..9 = epilogue (lane quarter = warp % 4). The PQ variant adds warps 10..13, which decode
// uint8 codes through a shared-memory fp16 codebook into the D stages instead of a TMA load; the
// residual variant adds warps 10..17, which rebuild residual-compressed tokens (centroid row +
// bucket weights, gathered one tile ahead into a shared-memory ring) into the D stages.
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "tms_device.cuh"
#include "tms_internal.h"

namespace tms {

namespace {

constexpr int kThreads = 320;    // 2 control warps + 8 epilogue warps
constexpr int kPqThreadsMma = 448;  // + 4 decoder warps (PQ variant)
// residual variant: RES decoder warps after the 10 warps of the dense kernel
constexpr int kResDecWarps = 8;
constexpr int res_threads(int res_warps) { return (10 + res_warps) * 32; }
constexpr int kDecodeWarp0 = 10;
constexpr int kEpiWarps = 8;
// Named barriers (0 is __syncthreads): each id belongs to one fixed group of warps.
constexpr int kBarEpilogue = 1;    // the 8 epilogue warps (column-split mode)
constexpr int kBarResDecode = 2;   // the residual decoder warps
constexpr int kQTileRows = 128;
constexpr uint32_t kQChunkBytes = kQTileRows * 128;  // one 128-row x 128-byte K chunk of Q
constexpr float kNegInf = -__builtin_huge_valf();

struct DenseArgs {
  DocLayout docs;
  float* out;
  uint32_t* err;
  uint64_t timeout_ns;
  int n_chunks_total;  // 32-row query chunks over all queries
  int nchunk;          // chunks per query
  int nq;
  int n_mtiles;
  int G;         // M tiles per CTA group
  int n_groups;  // CTA groups along the query dimension
  int n_ranges;  // token ranges along the document dimension
  int kc;        // 128-byte K chunks per row (ceil(d * esize / 128))
  int stages;
  int out_mode;
  uint32_t ab_format;  // MMA operand format: 0 = f16, 1 = bf16, 2 = tf32
  // PQ variant: D rows are decoded from codes (n_tokens, M) through codebook (M, K, dsub)
  const uint8_t* codes;
  int64_t n_code_rows;  // PQ variant: rows of codes; its token range is clamped to them
  const void* codebook;
  int cb_dtype, pq_M, pq_K, pq_dsub;
  uint32_t cb_bytes;   // fp16 codebook bytes staged in shared memory (0 for the dense kernel)
  // Residual-compressed tokens (the PQ variant's decoders in residual mode, res_nbits != 0):
  // token = centroids[res_codes[t]] + bucket_weights[per-dimension nbits index from res_bits],
  // optionally L2-normalised; the fp32 bucket weights take the codebook's shared-memory slot.
  const __half* res_centroids;  // (res_ncent, d) fp16
  const int32_t* res_codes;     // (n_tokens,)
  const uint8_t* res_bits;      // (n_tokens, d * res_nbits / 8)
  const float* res_bw;          // (1 << res_nbits,)
  int64_t res_ncent;
  int res_nbits;      // 0: PQ mode; 1, 2 or 4: residual mode
  int res_normalize;
  int debug_flags;     // bit 0: producer issues no load (exercises the bounded waits)
};

// Shared-memory carve-up, identical on host and device. `split` (one query of <= 32 tokens) adds
// the exchange area of the column-split epilogue and drops the per-row carries.
struct SmemLayout {
  uint32_t q_off, stage_off, stage_bytes, bar_off, carry_off, x_off, cb_off, misc_off, total;
};
struct PartMeta {  // one epilogue warp's summary of its column part (split mode)
  int64_t head_doc;  // document whose end lies in the part (valid if has_b)
  int64_t end_doc, end_dend;  // walk state after the part
  int32_t has_b, pad;
};
__host__ __device__ inline SmemLayout dense_smem_layout(int TN, bool qres, int G, int kc,
                                                        int stages, bool split,
                                                        uint32_t cb_bytes = 0) {
  SmemLayout L;
  L.q_off = 0;
  const uint32_t q_bytes = qres ? static_cast<uint32_t>(G * kc) * kQChunkBytes : 0u;
  L.stage_off = q_bytes;
  L.stage_bytes = qres ? static_cast<uint32_t>(kc * TN * 128) : (kQChunkBytes + TN * 128u);
  L.bar_off = L.stage_off + static_cast<uint32_t>(stages) * L.stage_bytes;
  const uint32_t n_bars = 2u * stages + 2u * (512u / TN) + 2u;  // + accumulator slots, q, done
  L.carry_off = (L.bar_off + n_bars * 8u + 15u) & ~15u;
  L.x_off = L.carry_off + (split ? 0u : static_cast<uint32_t>(G) * kQTileRows * 4u);
  const uint32_t x_bytes =
      split ? 2u * (2u * kEpiWarps * 32u * 4u + kEpiWarps * static_cast<uint32_t>(sizeof(PartMeta)))
            : 0u;  // split mode: two buffers (tile parity)
  L.cb_off = (L.x_off + x_bytes + 15u) & ~15u;
  L.misc_off = (L.cb_off + cb_bytes + 15u) & ~15u;
  L.total = L.misc_off + 64u;
  return L;
}

struct RangeInfo {
  int64_t doc_lo, doc_hi, tok_lo, tok_hi;
};

__device__ __forceinline__ float u2f(uint32_t x) { return __uint_as_float(x); }

// Three-input fp32 max (PTX max.f32 with three sources, sm_100a).
__device__ __forceinline__ float fmax3(float x, float y, float z) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(x), "f"(y), "f"(z));
  return r;
}

// max(acc, r[0..31]) with four independent chains.
__device__ __forceinline__ float max32(float acc, const uint32_t (&r)[32]) {
  float m[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) m[j] = fmax3(u2f(r[j]), u2f(r[j + 4]), u2f(r[j + 8]));
#pragma unroll
  for (int i = 12; i < 28; i += 8)
#pragma unroll
    for (int j = 0; j < 4; ++j) m[j] = fmax3(m[j], u2f(r[i + j]), u2f(r[i + 4 + j]));
#pragma unroll
  for (int j = 0; j < 4; ++j) m[j] = fmaxf(m[j], u2f(r[28 + j]));
  return fmax3(fmax3(acc, m[0], m[1]), m[2], m[3]);
}

// max(acc, r[lo..hi)) (acc when the range is empty).
__device__ __forceinline__ float range_max32(float acc, const uint32_t (&r)[32], int lo, int hi) {
  float m0 = acc, m1 = kNegInf;
  const uint32_t span = static_cast<uint32_t>(hi - lo);
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    const float a0 = static_cast<uint32_t>(i - lo) < span ? u2f(r[i]) : kNegInf;
    const float a1 = static_cast<uint32_t>(i + 1 - lo) < span ? u2f(r[i + 1]) : kNegInf;
    const float a2 = static_cast<uint32_t>(i + 2 - lo) < span ? u2f(r[i + 2]) : kNegInf;
    const float a3 = static_cast<uint32_t>(i + 3 - lo) < span ? u2f(r[i + 3]) : kNegInf;
    m0 = fmax3(m0, a0, a1);
    m1 = fmax3(m1, a2, a3);
  }
  return fmaxf(m0, m1);
}

// max(init, r[LO..HI)) over compile-time column ranges, two independent chains.
template <int LO, int HI>
__device__ __forceinline__ float cmax(float init, const uint32_t (&r)[32]) {
  float m0 = init, m1 = kNegInf;
#pragma unroll
  for (int i = LO; i < HI; i += 4) {
    if (i + 1 < HI) m0 = fmax3(m0, u2f(r[i]), u2f(r[i + 1]));
    else m0 = fmaxf(m0, u2f(r[i]));
    if (i + 3 < HI) m1 = fmax3(m1, u2f(r[i + 2]), u2f(r[i + 3]));
    else if (i + 2 < HI) m1 = fmaxf(m1, u2f(r[i + 2]));
  }
  return fmaxf(m0, m1);
}

// A 32-column block with one document boundary at column p (warp-uniform, 0 <= p < 32):
// acc = max(acc, r[0..p)) and the return value is max(r[p..32)). A jump over 32 straight-line
// variants costs one indirect branch instead of a select per column.
template <int P>
__device__ __forceinline__ float split_at(float& acc, const uint32_t (&r)[32]) {
  acc = cmax<0, P>(acc, r);
  return cmax<P, 32>(kNegInf, r);
}
__device__ __forceinline__ float split_max32(float& acc, const uint32_t (&r)[32], int p) {
  switch (p) {
#define TMS_SPLIT_CASE(n) case n: return split_at<n>(acc, r);
    TMS_SPLIT_CASE(0) TMS_SPLIT_CASE(1) TMS_SPLIT_CASE(2) TMS_SPLIT_CASE(3) TMS_SPLIT_CASE(4)
    TMS_SPLIT_CASE(5) TMS_SPLIT_CASE(6) TMS_SPLIT_CASE(7) TMS_SPLIT_CASE(8) TMS_SPLIT_CASE(9)
    TMS_SPLIT_CASE(10) TMS_SPLIT_CASE(11) TMS_SPLIT_CASE(12) TMS_SPLIT_CASE(13) TMS_SPLIT_CASE(14)
    TMS_SPLIT_CASE(15) TMS_SPLIT_CASE(16) TMS_SPLIT_CASE(17) TMS_SPLIT_CASE(18) TMS_SPLIT_CASE(19)
    TMS_SPLIT_CASE(20) TMS_SPLIT_CASE(21) TMS_SPLIT_CASE(22) TMS_SPLIT_CASE(23) TMS_SPLIT_CASE(24)
    TMS_SPLIT_CASE(25) TMS_SPLIT_CASE(26) TMS_SPLIT_CASE(27) TMS_SPLIT_CASE(28) TMS_SPLIT_CASE(29)
    TMS_SPLIT_CASE(30)
#undef TMS_SPLIT_CASE
    default: return split_at<31>(acc, r);
  }
}

// Residual decoding works from a two-slot ring of shared memory that the decoder warps fill one
// tile ahead with asynchronous copies, so the L2 gathers of centroid rows overlap the decoding of
// the previous tile instead of stalling it. Before the ring, a byte table: for each byte value,
// the bucket weights of the 8 / nbits dimensions that byte encodes (the first dimension in the
// byte's high bits).
constexpr int kResRing = 2;
struct ResLayout {
  uint32_t table_off, slot_off, slot_bytes, bits_off, pitch, rb, total;
};
__host__ __device__ inline ResLayout residual_layout(int d, int nb) {
  ResLayout R;
  R.pitch = static_cast<uint32_t>(2 * d);
  R.rb = static_cast<uint32_t>(d * nb / 8);
  R.table_off = 8u * kResRing;                                   // after the ring's mbarriers
  R.slot_off = (R.table_off + 256u * (8u / nb) * 4u + 127u) & ~127u;
  R.bits_off = 128u * R.pitch;                                  // 128-token tiles
  R.slot_bytes = (R.bits_off + 128u * R.rb + 127u) & ~127u;
  R.total = R.slot_off + kResRing * R.slot_bytes;
  return R;
}

// Adds the bucket weights of one 8-dimension unit (its NB residual bytes, little-endian in
// `bits`) to the unit's centroid values; x[k] holds dimensions 2k and 2k + 1 as an fp32 pair.
template <int NB>
__device__ __forceinline__ void residual_unit(const uint4& c, uint32_t bits, const float* table,
                                              uint64_t (&x)[4]) {
  const uint32_t cw[4] = {c.x, c.y, c.z, c.w};
  uint64_t w[4];
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const uint32_t v = (bits >> (8 * b)) & 0xffu;
    if (NB == 1) {
      const ulonglong2 w0 = reinterpret_cast<const ulonglong2*>(table)[2 * v];
      const ulonglong2 w1 = reinterpret_cast<const ulonglong2*>(table)[2 * v + 1];
      w[0] = w0.x; w[1] = w0.y; w[2] = w1.x; w[3] = w1.y;
    } else if (NB == 2) {
      const ulonglong2 wv = reinterpret_cast<const ulonglong2*>(table)[v];
      w[2 * b] = wv.x; w[2 * b + 1] = wv.y;
    } else {
      w[b] = reinterpret_cast<const unsigned long long*>(table)[v];
    }
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&cw[k]));
    x[k] = f2_add(f2_pack(f.x, f.y), w[k]);
  }
}

// The residual decoder role (DW warps, thread dt = 0 .. 32 DW - 1) for NB bits per dimension and D = 64 or
// 128 dimensions, compiled per (NB, D) so every loop below has a fixed trip count.
//
// Ring: tile i + 1's centroid rows and residual bytes are copied (cp.async) into ring slot
// (i + 1) % 2 while tile i is decoded from slot i % 2. Each warp gathers the centroid rows of its
// own 16 tokens in 16-byte pieces (consecutive lanes on consecutive pieces of a row; a row's
// centroid id comes from its token's lane by shuffle); the tile's residual bytes are contiguous
// and copied in 16-byte (or, for 8-byte rows or a residual buffer that is only 4-byte aligned,
// 4-byte) pieces. Every thread's copies arrive on the slot's mbarrier (256 arrivals).
//
// Decoding: in pass p (of 4), thread dt takes token 32 p + dt / 8 and its 16-byte units h and h + 8
// (h = dt % 8), so the eight lanes of a token read 128 contiguous bytes of the row (every bank once
// per phase) and add up the squared values for the norm with three shuffles. Values are
// centroid + bucket weight in fp32, scaled by the token's inverse norm, rounded once to fp16 and
// stored in the 128-byte-swizzle layout (unit u of row r at u ^ (r % 8)).
//
// A named barrier over the 256 decoder threads closes each tile (the slot it read is free again)
// and ORs the failure flag, so the four warps always leave the loop together; copies still in
// flight after a failure land before the CTA exits.
template <int NB, int D, int DW>
__device__ __forceinline__ void residual_decoders(const DenseArgs& a, uint8_t* smem, const SmemLayout& L,
                                                  uint32_t bar_s, int S, int64_t tok_lo, int64_t tok_hi,
                                                  volatile int* abort_flag, uint64_t tmo) {
  constexpr int UPP = D / 64;   // 16-byte units per thread per token
  constexpr int CPR = D / 8;    // 16-byte pieces per centroid row
  constexpr int RPS = 32 / CPR; // rows per warp-wide gather step
  constexpr int RB = D * NB / 8;  // residual bytes per token
  constexpr int PITCH = 2 * D;
  constexpr int NT = DW * 32;   // decoder threads
  constexpr int TPW = 128 / DW;  // tokens of a tile each warp gathers
  const int dt = static_cast<int>(threadIdx.x) - kDecodeWarp0 * 32;
  const int lane = dt & 31, tw = (dt >> 5) * TPW;
  const int tc = tw + (lane % TPW);  // the token whose centroid id this thread holds
  const ResLayout R = residual_layout(D, NB);
  uint8_t* cbase = smem + L.cb_off;
  const uint32_t ring_bar = smem_u32(cbase);
  const float* table = reinterpret_cast<const float*>(cbase + R.table_off);
  const bool w16 = (RB % 16 == 0) && (reinterpret_cast<uintptr_t>(a.res_bits) & 15) == 0;
  const int64_t ncent = a.res_ncent;
  const bool nrm = a.res_normalize != 0;
  const int64_t n_tiles = (tok_hi - tok_lo + 127) / 128;
  auto full_bar = [&](int s) { return bar_s + 8u * s; };
  auto empty_bar = [&](int s) { return bar_s + 8u * (S + s); };

  int32_t code_next = tok_lo + tc < tok_hi ? __ldg(a.res_codes + tok_lo + tc) : 0;
  auto issue = [&](int64_t j) {
    const int64_t t0 = tok_lo + 128 * j;
    const int sl = static_cast<int>(j % kResRing);
    const uint32_t slot = smem_u32(cbase + R.slot_off + sl * R.slot_bytes);
    int32_t c = code_next;
    code_next = t0 + 128 + tc < tok_hi ? __ldg(a.res_codes + t0 + 128 + tc) : 0;
    c = c < 0 ? 0 : (c >= ncent ? static_cast<int32_t>(ncent - 1) : c);  // never outside the table
    const int n = static_cast<int>(min(int64_t(128), tok_hi - t0));
    const int pc = lane % CPR;
#pragma unroll
    for (int m = 0; m < TPW / RPS; ++m) {
      const int tl = m * RPS + lane / CPR;  // token within the warp's TPW
      const int32_t cc = __shfl_sync(0xffffffffu, c, tl);
      if (tw + tl < n)
        cp_async16(slot + static_cast<uint32_t>((tw + tl) * PITCH + 16 * pc),
                   a.res_centroids + static_cast<int64_t>(cc) * D + 8 * pc);
    }
    const uint8_t* src = a.res_bits + t0 * RB;
    const uint32_t dst = slot + R.bits_off;
    if (RB % 16 == 0 && w16) {
      const int lim = n * (RB / 16);
#pragma unroll
      for (int q = 0; q < (8 * RB + NT - 1) / NT; ++q) {
        const int k = dt + NT * q;
        if (k < lim) cp_async16(dst + 16u * k, src + 16 * k);
      }
    } else {
      const int lim = n * (RB / 4);
#pragma unroll
      for (int q = 0; q < (32 * RB + NT - 1) / NT; ++q) {
        const int k = dt + NT * q;
        if (k < lim) cp_async4(dst + 4u * k, src + 4 * k);
      }
    }
    cp_async_mbar_arrive_noinc(ring_bar + 8u * sl);
  };

  auto decode = [&](const uint8_t* slot, int n_valid, uint8_t* stage) {
    const int tk = dt >> 3, h = dt & 7;
#pragma unroll 2
    for (int p = 0; p < 128 * 8 / NT; ++p) {
      const int r = (NT / 8) * p + tk;
      const uint8_t* crow = slot + r * PITCH;
      const uint8_t* brow = slot + R.bits_off + r * RB;
      uint64_t x[UPP][4];
#pragma unroll
      for (int i = 0; i < UPP; ++i) {
        const int u = h + 8 * i;
        const uint4 c = *reinterpret_cast<const uint4*>(crow + u * 16);
        uint32_t bits;
        if (NB == 4) bits = *reinterpret_cast<const uint32_t*>(brow + u * 4);
        else if (NB == 2) bits = *reinterpret_cast<const unsigned short*>(brow + u * 2);
        else bits = brow[u];
        residual_unit<NB>(c, bits, table, x[i]);
      }
      float scale = 1.0f;
      if (nrm) {
        uint64_t s0 = 0ull, s1 = 0ull;  // two pairs of partial sums of squares
#pragma unroll
        for (int i = 0; i < UPP; ++i)
#pragma unroll
          for (int k = 0; k < 4; k += 2) {
            s0 = f2_fma(x[i][k], x[i][k], s0);
            s1 = f2_fma(x[i][k + 1], x[i][k + 1], s1);
          }
        const float2 q = f2_unpack(f2_add(s0, s1));
        float ss = q.x + q.y;
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        ss += __shfl_xor_sync(0xffffffffu, ss, 4);
        scale = ss > 0.0f ? rsqrtf(ss) : 0.0f;
      }
      if (r < n_valid) {
        uint8_t* rowp = stage + r * 128;
        const uint32_t sw = static_cast<uint32_t>(r & 7);
#pragma unroll
        for (int i = 0; i < UPP; ++i) {
          const int u = h + 8 * i;
          const uint64_t sc2 = f2_pack(scale, scale);
          uint32_t pk[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 v = f2_unpack(f2_mul(x[i][k], sc2));
            const __half2 hv = __floats2half2_rn(v.x, v.y);
            pk[k] = *reinterpret_cast<const uint32_t*>(&hv);
          }
          *reinterpret_cast<uint4*>(rowp + (u >> 3) * (128 * 128) + (((static_cast<uint32_t>(u) & 7u) ^ sw) << 4)) =
              make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
    }
  };

  int s = 0;
  uint32_t ph = 0;
  bool ok = !(a.debug_flags & 1);
  int64_t issued = 0;
  if (ok && n_tiles > 0) {
    issue(0);
    issued = 1;
  }
  for (int64_t i = 0; ok && i < n_tiles; ++i) {
    if (i + 1 < n_tiles) {
      issue(i + 1);
      issued = i + 2;
    }
    int w = 0;
    if (lane == 0) w = mbar_wait(empty_bar(s), ph ^ 1u, abort_flag, tmo, a.err, 10);
    bool good = __shfl_sync(0xffffffffu, w, 0) != 0;
    const int sl = static_cast<int>(i % kResRing);
    if (good)
      good = mbar_wait(ring_bar + 8u * sl, static_cast<uint32_t>((i / kResRing) & 1), abort_flag, tmo,
                       a.err, 11);
    good = __all_sync(0xffffffffu, good);
    if (good) {
      const int64_t t0 = tok_lo + 128 * i;
      decode(cbase + R.slot_off + sl * R.slot_bytes, static_cast<int>(min(int64_t(128), tok_hi - t0)),
             smem + L.stage_off + static_cast<size_t>(s) * L.stage_bytes);
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core's reads
      __syncwarp();
      if (lane == 0) mbar_arrive(full_bar(s));
    }
    if (++s == S) { s = 0; ph ^= 1u; }
    ok = !named_barrier_or(kBarResDecode, NT, !good);
  }
  cp_async_wait_all();
  for (int64_t j = issued >= 2 ? issued - 2 : 0; !ok && j < issued; ++j) {
    const uint32_t bar = ring_bar + 8u * static_cast<uint32_t>(j % kResRing);
    const uint32_t par = static_cast<uint32_t>((j / kResRing) & 1);
    const uint64_t tw0 = globaltimer_ns();
    while (!mbar_try_wait(bar, par) && globaltimer_ns() - tw0 < tmo) {
    }
  }
}

template <int TN, bool QRES, bool TF32, bool PQ, int RES = 0>
__global__ void __launch_bounds__(RES ? res_threads(RES) : PQ ? kPqThreadsMma : kThreads, 1)
    dense_maxsim_kernel(const __grid_constant__ CUtensorMap qmap,
                        const __grid_constant__ CUtensorMap dmap, const DenseArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  // one query tile (1-4 chunks): column-split epilogue over nc = 1, 2 or 4 replicated chunks
  const bool split = a.n_mtiles == 1;
  const int split_nc = a.n_chunks_total == 1 ? 1 : a.n_chunks_total == 2 ? 2 : 4;
  const SmemLayout L = dense_smem_layout(TN, QRES, a.G, a.kc, a.stages, split, a.cb_bytes);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t q_s = sbase + L.q_off;
  const uint32_t st_s = sbase + L.stage_off;
  const uint32_t bar_s = sbase + L.bar_off;
  const int S = a.stages;
  auto full_bar = [&](int s) { return bar_s + 8u * s; };
  auto empty_bar = [&](int s) { return bar_s + 8u * (S + s); };
  constexpr int NSLOT = 512 / TN;  // TMEM accumulator slots (all 512 columns)
  auto accf_bar = [&](int b) { return bar_s + 8u * (2 * S + b); };
  auto acce_bar = [&](int b) { return bar_s + 8u * (2 * S + NSLOT + b); };
  const uint32_t qfull_bar = bar_s + 8u * (2 * S + 2 * NSLOT);
  const uint32_t done_bar = bar_s + 8u * (2 * S + 2 * NSLOT + 1);
  float* carry = reinterpret_cast<float*>(smem + L.carry_off);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.misc_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.misc_off + 4);
  volatile int* never_flag = reinterpret_cast<volatile int*>(smem + L.misc_off + 8);  // stays 0
  RangeInfo* rinfo = reinterpret_cast<RangeInfo*>(smem + L.misc_off + 16);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int range = blockIdx.x / a.n_groups;
  const int group = blockIdx.x - range * a.n_groups;
  const int m_first = group * a.G;
  const int g_this = min(a.G, a.n_mtiles - m_first);
  // rows mode: the two epilogue groups take alternate query tiles (m parity). Only with an even
  // number of tiles per CTA: then the slot of unit u = t*g_this + m has the parity of m, so every
  // TMEM slot belongs to one group, which waits on each of its phases in order (with an odd count
  // a group would skip phases and a parity wait could match a stale completion two phases back).
  const bool two_groups = !split && g_this >= 2 && (g_this & 1) == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), RES ? RES : PQ ? 4 : 1);  // one arrival per decoder warp
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < NSLOT; ++b) {
      mbar_init(accf_bar(b), 1);
      mbar_init(acce_bar(b), split ? kEpiWarps : 4);
    }
    mbar_init(qfull_bar, 1);
    mbar_init(done_bar, 1);
    if (RES)  // residual ring slots: one cp.async arrival per decoder thread
      for (int b = 0; b < kResRing; ++b) mbar_init(smem_u32(smem + L.cb_off) + 8u * b, RES * 32);
    *abort_flag = (smem_u32(smem) & 1023u) ? 1 : 0;  // SWIZZLE_128B needs a 1024-aligned base
    *never_flag = 0;
    if (*abort_flag) atomicCAS(a.err, 0u, kDevErrTimeout | 15u);
    fence_mbar_init();
  }
  if (warp == 0) {
    // Cut this CTA's token range at document boundaries.
    const int64_t t_first = a.docs.start(0);
    const int64_t t_last = a.docs.start(a.docs.n_docs);
    const int64_t span = t_last - t_first;
    const int64_t tgt_lo = t_first + span * range / a.n_ranges;
    const int64_t tgt_hi = t_first + span * (range + 1) / a.n_ranges;
    const int64_t doc_lo = (range == 0) ? 0 : warp_lower_bound(a.docs, tgt_lo);
    const int64_t doc_hi =
        (range == a.n_ranges - 1) ? a.docs.n_docs : warp_lower_bound(a.docs, tgt_hi);
    if (lane == 0) {
      rinfo->doc_lo = doc_lo;
      rinfo->doc_hi = doc_hi;
      rinfo->tok_lo = a.docs.start(doc_lo);
      rinfo->tok_hi = (doc_hi > doc_lo) ? a.docs.start(doc_hi) : a.docs.start(doc_lo);
      if (PQ) {  // decoders read codes rows [tok_lo, tok_hi): keep them inside the array
        rinfo->tok_lo = max(min(rinfo->tok_lo, a.n_code_rows), int64_t(0));
        rinfo->tok_hi = max(min(rinfo->tok_hi, a.n_code_rows), rinfo->tok_lo);
      }
      prefetch_tmap(&dmap);
      prefetch_tmap(&qmap);
    }
  }
  if (PQ) {  // stage the codebook in shared memory as fp16 (every thread helps)
    __half* cbs = reinterpret_cast<__half*>(smem + L.cb_off);
    if (RES) {
      // byte table: entry v, field q = the weight of the bucket whose index has bit k equal to
      // bit (7 - q * nbits - k) of v (the packing is MSB-first, lowest index bit first)
      const int nb = a.res_nbits, per = 8 / nb;
      const ResLayout R = residual_layout(a.kc * 64, nb);
      float* table = reinterpret_cast<float*>(smem + L.cb_off + R.table_off);
      for (int i = threadIdx.x; i < 256 * per; i += blockDim.x) {
        const int v = i / per, q = i - v * per;
        int idx = 0;
        for (int k = 0; k < nb; ++k) idx |= ((v >> (7 - q * nb - k)) & 1) << k;
        table[i] = a.res_bw[idx];
      }
    }
    const int n = a.res_nbits ? 0 : a.pq_M * a.pq_K * a.pq_dsub;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      float v;
      if (a.cb_dtype == TMS_F16) v = __half2float(reinterpret_cast<const __half*>(a.codebook)[i]);
      else if (a.cb_dtype == TMS_BF16) v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.codebook)[i]);
      else v = reinterpret_cast<const float*>(a.codebook)[i];
      cbs[i] = __float2half_rn(v);
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint32_t tmem_base = *tmem_slot;
  const int64_t doc_lo = rinfo->doc_lo, doc_hi = rinfo->doc_hi;
  const int64_t tok_lo = rinfo->tok_lo, tok_hi = rinfo->tok_hi;
  const uint64_t tmo = a.timeout_ns;
  const bool dead = *abort_flag != 0;

  if (dead) {
    // misaligned shared memory: no role runs (the error word says why)
  } else if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0 && !(a.debug_flags & 1)) {
      const uint64_t pol_d = (a.n_groups > 1) ? policy_evict_normal() : policy_evict_first();
      const uint64_t pol_q = policy_evict_last();
      const int cw = TF32 ? 32 : 64;  // elements per 128-byte chunk
      if (QRES && tok_hi > tok_lo) {
        mbar_arrive_expect_tx(qfull_bar, static_cast<uint32_t>(g_this * a.kc) * kQChunkBytes);
        for (int m = 0; m < g_this; ++m)
          for (int c = 0; c < a.kc; ++c)
            tma_load_2d(q_s + static_cast<uint32_t>(m * a.kc + c) * kQChunkBytes, &qmap, qfull_bar,
                        c * cw, (m_first + m) * kQTileRows, pol_q);
      }
      int s = 0;
      uint32_t ph = 0;
      uint32_t armed = 0, armed_par = 0;  // per stage: a load was issued, and its phase parity
      auto arm = [&](int st_i, uint32_t par, uint32_t bytes) {
        mbar_arrive_expect_tx(full_bar(st_i), bytes);
        armed |= 1u << st_i;
        armed_par = (armed_par & ~(1u << st_i)) | (par << st_i);
      };
      bool ok = !PQ;  // the PQ variant's D stages are filled by the decoder warps
      for (int64_t t0 = tok_lo; ok && t0 < tok_hi; t0 += TN) {
        if (QRES) {
          if (!(ok = mbar_wait(empty_bar(s), ph ^ 1u, abort_flag, tmo, a.err, 1))) break;
          arm(s, ph, static_cast<uint32_t>(a.kc * TN * 128));
          const uint32_t st = st_s + static_cast<uint32_t>(s) * L.stage_bytes;
          for (int c = 0; c < a.kc; ++c)
            tma_load_2d(st + static_cast<uint32_t>(c * TN * 128), &dmap, full_bar(s), c * cw,
                        static_cast<int32_t>(t0), pol_d);
          if (++s == S) { s = 0; ph ^= 1u; }
        } else {
          for (int m = 0; ok && m < g_this; ++m) {
            for (int c = 0; c < a.kc; ++c) {
              if (!(ok = mbar_wait(empty_bar(s), ph ^ 1u, abort_flag, tmo, a.err, 2))) break;
              arm(s, ph, kQChunkBytes + TN * 128u);
              const uint32_t st = st_s + static_cast<uint32_t>(s) * L.stage_bytes;
              tma_load_2d(st, &qmap, full_bar(s), c * cw, (m_first + m) * kQTileRows, pol_q);
              tma_load_2d(st + kQChunkBytes, &dmap, full_bar(s), c * cw, static_cast<int32_t>(t0),
                          pol_d);
              if (++s == S) { s = 0; ph ^= 1u; }
            }
          }
        }
      }
      if (*abort_flag) {
        // A wait gave up somewhere in the CTA: before the CTA exits, let every copy this thread
        // issued land in shared memory (each bounded by the wait limit on its own).
        if (QRES && tok_hi > tok_lo) mbar_wait(qfull_bar, 0, never_flag, tmo, a.err, 11);
        for (int st_i = 0; st_i < S; ++st_i)
          if (armed & (1u << st_i)) mbar_wait(full_bar(st_i), (armed_par >> st_i) & 1u, never_flag, tmo, a.err, 12);
      }
    }
  } else if (PQ && RES && warp >= kDecodeWarp0) {
    // ------------------------------------------------------------------ residual decoders
    const int nb = a.res_nbits;
    if (a.kc == 2) {
      if (nb == 2) residual_decoders<2, 128, (RES > 0 ? RES : 4)>(a, smem, L, bar_s, S, tok_lo, tok_hi, abort_flag, tmo);
      else if (nb == 1) residual_decoders<1, 128, (RES > 0 ? RES : 4)>(a, smem, L, bar_s, S, tok_lo, tok_hi, abort_flag, tmo);
      else residual_decoders<4, 128, (RES > 0 ? RES : 4)>(a, smem, L, bar_s, S, tok_lo, tok_hi, abort_flag, tmo);
    } else {
      if (nb == 2) residual_decoders<2, 64, (RES > 0 ? RES : 4)>(a, smem, L, bar_s, S, tok_lo, tok_hi, abort_flag, tmo);
      else if (nb == 1) residual_decoders<1, 64, (RES > 0 ? RES : 4)>(a, smem, L, bar_s, S, tok_lo, tok_hi, abort_flag, tmo);
      else residual_decoders<4, 64, (RES > 0 ? RES : 4)>(a, smem, L, bar_s, S, tok_lo, tok_hi, abort_flag, tmo);
    }
  } else if (PQ && !RES && warp >= kDecodeWarp0) {
    // ------------------------------------------------------------------ PQ decoders
    // Row r of a D stage = token t0 + r rebuilt from its M codes: codebook row (m, code) is
    // dsub fp16 values = dsub/8 16-byte units, placed at columns m*dsub.. of the row in the
    // 128-byte-swizzle layout the MMA descriptors expect (unit u of row r at u ^ (r % 8)).
    const __half* cbs = reinterpret_cast<const __half*>(smem + L.cb_off);
    const int dt = threadIdx.x - kDecodeWarp0 * 32;  // 0..127
    const int M = a.pq_M, K = a.pq_K, dsub = a.pq_dsub;
    const bool m16 = (M == 16) && ((reinterpret_cast<uintptr_t>(a.codes) & 15) == 0);
    int s = 0;
    uint32_t ph = 0;
    bool ok = !(a.debug_flags & 1);
    constexpr int TPT = TN / 128;  // tokens per decoder thread per tile
    // Codes of the common shape are prefetched two tiles ahead in registers, so the HBM latency of
    // a tile's codes overlaps the decoding of the tiles before it.
    auto load_codes = [&](int64_t t0, uint4 (&c)[TPT]) {
#pragma unroll
      for (int i = 0; i < TPT; ++i) {
        const int64_t tok = t0 + dt + 128 * i;
        c[i] = (m16 && dsub == 8 && tok < tok_hi)
                   ? __ldg(reinterpret_cast<const uint4*>(a.codes + tok * 16))
                   : make_uint4(0, 0, 0, 0);
      }
    };
    uint4 c_cur[TPT], c_n1[TPT], c_n2[TPT];
    load_codes(tok_lo, c_n1);
    load_codes(tok_lo + TN, c_n2);
    for (int64_t t0 = tok_lo; ok && t0 < tok_hi; t0 += TN) {
#pragma unroll
      for (int i = 0; i < TPT; ++i) {
        c_cur[i] = c_n1[i];
        c_n1[i] = c_n2[i];
      }
      load_codes(t0 + 2 * TN, c_n2);
      int w = 0;
      if (lane == 0) w = mbar_wait(empty_bar(s), ph ^ 1u, abort_flag, tmo, a.err, 9);
      if (!(ok = __shfl_sync(0xffffffffu, w, 0) != 0)) break;
      uint8_t* st = smem + L.stage_off + static_cast<size_t>(s) * L.stage_bytes;
#pragma unroll
      for (int i = 0; i < TPT; ++i) {
        const int r = dt + 128 * i;
        const int64_t tok = t0 + r;
        if (tok >= tok_hi) continue;  // columns past the range are never read by the epilogue
        const uint8_t* crow = a.codes + tok * M;
        uint8_t* rowp = st + r * 128;
        const uint32_t sw = static_cast<uint32_t>(r & 7);
        if (m16 && dsub == 8) {
          // common shape (M = 16, dsub = 8, d = 128): 16 unrolled 16-byte copies
          const uint32_t cw[4] = {c_cur[i].x, c_cur[i].y, c_cur[i].z, c_cur[i].w};
#pragma unroll
          for (int m = 0; m < 16; ++m) {
            uint32_t code = (cw[m >> 2] >> (8 * (m & 3))) & 0xffu;
            code = min(code, static_cast<uint32_t>(K - 1));  // never read past the codebook
            const uint4 v = *reinterpret_cast<const uint4*>(cbs + (m * K + code) * 8);
            *reinterpret_cast<uint4*>(rowp + (m >> 3) * (TN * 128) + (((m & 7) ^ sw) << 4)) = v;
          }
        } else {
          for (int m = 0; m < M; ++m) {
            const uint32_t code = min(static_cast<uint32_t>(__ldg(crow + m)), static_cast<uint32_t>(K - 1));
            const uint4* src = reinterpret_cast<const uint4*>(cbs + (m * K + code) * dsub);
            for (int h = 0; h < dsub; h += 8) {
              const int col = m * dsub + h;
              const uint32_t u = static_cast<uint32_t>((col & 63) >> 3);
              *reinterpret_cast<uint4*>(rowp + (col >> 6) * (TN * 128) + ((u ^ sw) << 4)) = src[h >> 3];
            }
          }
        }
      }
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core's reads
      __syncwarp();
      if (lane == 0) mbar_arrive(full_bar(s));
      if (++s == S) { s = 0; ph ^= 1u; }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc(128, TN, a.ab_format);
      bool ok = true;
      if (QRES && tok_hi > tok_lo) ok = mbar_wait(qfull_bar, 0, abort_flag, tmo, a.err, 3);
      int s = 0;
      uint32_t ph = 0, u = 0;
      for (int64_t t0 = tok_lo; ok && t0 < tok_hi; t0 += TN) {
        if (QRES) {
          if (!(ok = mbar_wait(full_bar(s), ph, abort_flag, tmo, a.err, 4))) break;
          tc_fence_after();
        }
        for (int m = 0; ok && m < g_this; ++m, ++u) {
          const uint32_t slot = u % NSLOT;
          if (!(ok = mbar_wait(acce_bar(slot), ((u / NSLOT) & 1u) ^ 1u, abort_flag, tmo, a.err, 5)))
            break;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + slot * TN;
          for (int c = 0; c < a.kc; ++c) {
            uint32_t a_base, b_base;
            if (QRES) {
              a_base = q_s + static_cast<uint32_t>(m * a.kc + c) * kQChunkBytes;
              b_base = st_s + static_cast<uint32_t>(s) * L.stage_bytes +
                       static_cast<uint32_t>(c * TN * 128);
            } else {
              if (!(ok = mbar_wait(full_bar(s), ph, abort_flag, tmo, a.err, 6))) break;
              tc_fence_after();
              a_base = st_s + static_cast<uint32_t>(s) * L.stage_bytes;
              b_base = a_base + kQChunkBytes;
            }
            // descriptors of the 4 K slices of this chunk: the start address field counts
            // 16-byte units, so each 32-byte K step adds 2
            const uint64_t ad0 = sw128_kmajor_desc(a_base);
            const uint64_t bd0 = sw128_kmajor_desc(b_base);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              if (TF32)
                mma_tf32(d_tmem, ad0 + 2u * k, bd0 + 2u * k, idesc, (c | k) != 0);
              else
                mma_f16(d_tmem, ad0 + 2u * k, bd0 + 2u * k, idesc, (c | k) != 0);
            }
            if (!QRES) {
              mma_commit(empty_bar(s));
              if (++s == S) { s = 0; ph ^= 1u; }
            }
          }
          if (!ok) break;
          mma_commit(accf_bar(slot));
        }
        if (QRES && ok) {
          mma_commit(empty_bar(s));
          if (++s == S) { s = 0; ph ^= 1u; }
        }
      }
      // Make sure every MMA this thread issued has landed before TMEM is released.
      mma_commit(done_bar);
      mbar_wait(done_bar, 0, abort_flag, tmo, a.err, 7);
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int ew = warp - 2;  // epilogue warp 0..7
    const int eg = ew >> 2;   // epilogue group (rows mode)
    const int lg = warp & 3;  // TMEM lane quarter this warp may access
    const int row = lg * 32 + lane;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(lg * 32) << 16);
    const DocLayout docs = a.docs;
    // Document ends are fetched 32 at a time (one coalesced load per warp) and handed out with
    // shuffles, so walking the document boundaries costs one global load per 32 documents.
    int64_t e_base = INT64_MIN / 2;  // first document whose end is cached in `ends`
    int64_t ends = 0;
    auto doc_end = [&](int64_t dd) -> int64_t {
      if (dd >= doc_hi) return INT64_MAX;
      int64_t idx = dd - e_base;
      if (idx < 0 || idx >= 32) {
        e_base = dd;
        const int64_t j = dd + 1 + lane;
        ends = (j <= docs.n_docs) ? docs.start(j) : INT64_MAX;
        idx = 0;
      }
      return __shfl_sync(0xffffffffu, ends, static_cast<int>(idx));
    };
    auto emit = [&](int chunk, int64_t dd, float rm) {
      const int q = chunk / a.nchunk;
      const int rq = (chunk - q * a.nchunk) * 32 + lane;
      const bool valid = rq < a.nq;
      if (a.out_mode == TMS_OUT_SCORE) {
        const float s = warp_sum(valid ? rm : 0.0f);
        if (lane == 0) a.out[static_cast<int64_t>(chunk) * docs.n_docs + dd] = s;
      } else if (valid) {
        a.out[(static_cast<int64_t>(q) * docs.n_docs + dd) * a.nq + rq] = rm;
      }
    };
    auto wait_full = [&](uint32_t slot, uint32_t uu) -> bool {
      int w = 0;
      if (lane == 0) w = mbar_wait(accf_bar(slot), (uu / NSLOT) & 1u, abort_flag, tmo, a.err, 8);
      return __shfl_sync(0xffffffffu, w, 0) != 0;
    };

    int64_t doc = doc_lo;
    int64_t dend = doc_end(doc);
    uint32_t u = 0;
    bool ok = true;
    if (split && split_nc == 1) {
      // ---- split mode, single chunk (the single-query hot path). A specialisation of the
      // general column-split branch below (nc = 1, one 32-column load per part): kept separate
      // because the general loop measured 15-20% slower here.
      // One query replicated in all four lane quarters; warp ew owns columns
      // [32*ew, 32*ew+32) of every tile. Documents wholly inside a part are emitted by its warp;
      // the part's first (head) and last (tail) partial maxima go through shared memory and
      // warp 0 of the epilogue chains them across parts and tiles.
      // exchange area, double-buffered by tile parity: a warp writes tile t+2's buffer only
      // after passing tile t+1's barrier, which the combine warp reaches after combining tile t
      constexpr uint32_t kXBuf = 2u * kEpiWarps * 32u * 4u + kEpiWarps * sizeof(PartMeta);
      constexpr int kParts = TN / 32;
      float running = kNegInf;  // combine warp: max of the document open at the last part's end
      for (int64_t t0 = tok_lo; ok && t0 < tok_hi; t0 += TN, ++u) {
        const uint32_t slot = u % NSLOT;
        float* xhead = reinterpret_cast<float*>(smem + L.x_off + (u & 1u) * kXBuf);
        float* xtail = xhead + kEpiWarps * 32;
        PartMeta* xmeta = reinterpret_cast<PartMeta*>(xtail + kEpiWarps * 32);
        const bool w_ok = wait_full(slot, u);
        tc_fence_after();
        const int ncol = (tok_hi - t0 < TN) ? static_cast<int>(tok_hi - t0) : TN;
        const int pc0 = 32 * ew;
        float head = kNegInf, tail = kNegInf;
        int has_b = 0;
        int64_t head_doc = -1, dd = doc, de = dend;
        if (w_ok && ew < kParts && pc0 < ncol) {
          uint32_t r[32];
          tmem_ld32_async(t_lane + slot * TN + pc0, r);
          tmem_wait_ld32(r);
          {
            auto rel = [&](int64_t e) -> int {
              const int64_t x = e - t0;
              return x > 4 * TN ? 4 * TN : static_cast<int>(x);
            };
            int dcol = rel(de);
            while (dcol < pc0) {  // documents that end before this part belong to earlier parts
              ++dd;
              de = doc_end(dd);
              dcol = rel(de);
            }
            const int n = (ncol - pc0 < 32) ? ncol - pc0 : 32;
            float rm = kNegInf;
            int lo = 0;
            while (true) {
              const int hi = (dcol - pc0 < n) ? dcol - pc0 : n;
              rm = (lo == 0 && hi == 32) ? max32(rm, r) : range_max32(rm, r, lo, hi);
              if (dcol - pc0 >= n) break;
              if (!has_b) {
                head = rm;
                head_doc = dd;
                has_b = 1;
              } else {
                emit(0, dd, rm);
              }
              rm = kNegInf;
              ++dd;
              de = doc_end(dd);
              dcol = rel(de);
              lo = hi;
            }
            if (has_b) tail = rm; else head = rm;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acce_bar(slot));  // this warp is done with the TMEM slot
        xhead[ew * 32 + lane] = head;
        xtail[ew * 32 + lane] = tail;
        if (lane == 0) {
          xmeta[ew].head_doc = head_doc;
          xmeta[ew].has_b = has_b;
          xmeta[ew].end_doc = dd;
          xmeta[ew].end_dend = de;
        }
        // all eight warps agree on whether every wait succeeded before anyone waits again
        uint32_t all_ok;
        asm volatile(
            "{\n\t.reg .pred p, q;\n\t"
            "setp.ne.u32 p, %1, 0;\n\t"
            "bar.red.and.pred q, %3, %2, p;\n\t"
            "selp.u32 %0, 1, 0, q;\n\t}\n"
            : "=r"(all_ok)
            : "r"(static_cast<uint32_t>(w_ok)), "n"(kEpiWarps * 32), "n"(kBarEpilogue)
            : "memory");
        if (!(ok = all_ok != 0)) break;
        const int n_parts = (ncol + 31) / 32;
        {
          if (ew == 0) {
            for (int pp = 0; pp < n_parts; ++pp) {
              running = fmaxf(running, xhead[pp * 32 + lane]);
              if (xmeta[pp].has_b) {
                emit(0, xmeta[pp].head_doc, running);
                running = xtail[pp * 32 + lane];
              }
            }
          }
          doc = xmeta[n_parts - 1].end_doc;
          dend = xmeta[n_parts - 1].end_dend;
        }
      }
      if (ok && ew == 0) {
        for (int64_t dd = doc; dd < doc_hi; ++dd) {
          emit(0, dd, running);
          running = kNegInf;
        }
      }
    } else if (split) {
      // ---- column-split mode (one query tile holding nc = 1, 2 or 4 chunks): the pack kernel
      // replicates the chunks over the four lane quarters (quarter lq holds chunk lq % nc), so
      // W = 8 / nc warps can read each chunk; warp ew (lane quarter lg = (ew + 2) & 3) takes part
      // p = ew / nc, columns [p*PC, p*PC + PC) of every tile of chunk c = lg % nc. The owner of
      // part p of chunk c is warp ew = p*nc + ((c - 2) & (nc - 1)). Documents wholly inside a part are
      // emitted by its warp; the part's head (max up to its first document end) and tail (max
      // after its last) go through shared memory, and the chunk's part-0 warp chains them across
      // parts and tiles.
      // exchange area, double-buffered by tile parity: a warp writes tile t+2's buffer only
      // after passing tile t+1's barrier, which the combine warps reach after combining tile t
      constexpr uint32_t kXBuf = 2u * kEpiWarps * 32u * 4u + kEpiWarps * sizeof(PartMeta);
      const int nc = split_nc;
      const int c = lg % nc;  // this warp's lane quarter holds chunk c
      const int pw = ew / nc;
      const int W = (8 / nc < TN / 32) ? 8 / nc : TN / 32;  // parts per chunk (>= 32 columns)
      const int PC = TN / W;
      const bool chunk_ok = c < a.n_chunks_total;
      float running = kNegInf;  // combine warp: max of the chunk's document open at the tile end
      for (int64_t t0 = tok_lo; ok && t0 < tok_hi; t0 += TN, ++u) {
        const uint32_t slot = u % NSLOT;
        float* xhead = reinterpret_cast<float*>(smem + L.x_off + (u & 1u) * kXBuf);
        float* xtail = xhead + kEpiWarps * 32;
        PartMeta* xmeta = reinterpret_cast<PartMeta*>(xtail + kEpiWarps * 32);
        const bool w_ok = wait_full(slot, u);
        tc_fence_after();
        const int ncol = (tok_hi - t0 < TN) ? static_cast<int>(tok_hi - t0) : TN;
        const int pc0 = pw * PC;
        float head = kNegInf, tail = kNegInf;
        int has_b = 0;
        int64_t head_doc = -1, dd = doc, de = dend;
        if (w_ok && chunk_ok && pw < W && pc0 < ncol) {
          auto rel = [&](int64_t e) -> int {
            const int64_t x = e - t0;
            return x > 4 * TN ? 4 * TN : static_cast<int>(x);
          };
          int dcol = rel(de);
          while (dcol < pc0) {  // documents that end before this part belong to earlier parts
            ++dd;
            de = doc_end(dd);
            dcol = rel(de);
          }
          const int pend = (ncol < pc0 + PC) ? ncol : pc0 + PC;
          float rm = kNegInf;
          auto reduce32 = [&](const uint32_t(&v)[32], int cb) {
            if (dcol >= cb + 32 && pend >= cb + 32) {
              rm = max32(rm, v);  // the whole block lies in the open document
            } else {
              const int n = (pend - cb < 32) ? pend - cb : 32;
              int lo = 0;
              while (true) {
                const int hi = (dcol - cb < n) ? dcol - cb : n;
                rm = range_max32(rm, v, lo, hi);
                if (dcol - cb >= n) break;
                if (!has_b) {
                  head = rm;
                  head_doc = dd;
                  has_b = 1;
                } else {
                  emit(c, dd, rm);
                }
                rm = kNegInf;
                ++dd;
                de = doc_end(dd);
                dcol = rel(de);
                lo = hi;
              }
            }
          };
          const uint32_t tbase = t_lane + slot * TN + pc0;
          if (PC == 32) {
            // one 32-column block per part (single query): one load, straight-line reduction
            uint32_t r[32];
            tmem_ld32_async(tbase, r);
            tmem_wait_ld32(r);
            const int n = pend - pc0;
            int lo = 0;
            while (true) {
              const int hi = (dcol - pc0 < n) ? dcol - pc0 : n;
              rm = (lo == 0 && hi == 32) ? max32(rm, r) : range_max32(rm, r, lo, hi);
              if (dcol - pc0 >= n) break;
              if (!has_b) {
                head = rm;
                head_doc = dd;
                has_b = 1;
              } else {
                emit(c, dd, rm);
              }
              rm = kNegInf;
              ++dd;
              de = doc_end(dd);
              dcol = rel(de);
              lo = hi;
            }
          } else {
          // 32-column TMEM loads, double-buffered (block b+1 in flight while b is reduced)
          uint32_t ra[32], rb[32];
          tmem_ld32_async(tbase, ra);
#pragma unroll
          for (int bk = 0; bk < 4; ++bk) {
            uint32_t(&cur)[32] = (bk & 1) ? rb : ra;
            uint32_t(&nxt)[32] = (bk & 1) ? ra : rb;
            const int cb = pc0 + 32 * bk;
            if (32 * bk < PC && cb < pend) {
              tmem_wait_ld32(cur);
              if (32 * (bk + 1) < PC && cb + 32 < pend) tmem_ld32_async(tbase + 32 * (bk + 1), nxt);
              reduce32(cur, cb);
            }
          }
          }
          if (has_b) tail = rm; else head = rm;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acce_bar(slot));  // this warp is done with the TMEM slot
        xhead[ew * 32 + lane] = head;
        xtail[ew * 32 + lane] = tail;
        if (lane == 0) {
          xmeta[ew].head_doc = head_doc;
          xmeta[ew].has_b = has_b;
          xmeta[ew].end_doc = dd;
          xmeta[ew].end_dend = de;
        }
        // all eight warps agree on whether every wait succeeded before anyone waits again
        uint32_t all_ok;
        asm volatile(
            "{\n\t.reg .pred p, q;\n\t"
            "setp.ne.u32 p, %1, 0;\n\t"
            "bar.red.and.pred q, %3, %2, p;\n\t"
            "selp.u32 %0, 1, 0, q;\n\t}\n"
            : "=r"(all_ok)
            : "r"(static_cast<uint32_t>(w_ok)), "n"(kEpiWarps * 32), "n"(kBarEpilogue)
            : "memory");
        if (!(ok = all_ok != 0)) break;
        const int n_parts = (ncol + PC - 1) / PC;
        {
          if (pw == 0 && chunk_ok) {
            for (int pp = 0; pp < n_parts; ++pp) {
              const int xe = nc * pp + ((c - 2) & (nc - 1));  // the warp owning part pp of chunk c
              running = fmaxf(running, xhead[xe * 32 + lane]);
              if (xmeta[xe].has_b) {
                emit(c, xmeta[xe].head_doc, running);
                running = xtail[xe * 32 + lane];
              }
            }
          }
          // the document walk is the same for every chunk: take it from chunk 0's last part
          const int xl = nc * (n_parts - 1) + ((0 - 2) & (nc - 1));
          doc = xmeta[xl].end_doc;
          dend = xmeta[xl].end_dend;
        }
      }
      if (ok && pw == 0 && chunk_ok) {
        for (int64_t dd = doc; dd < doc_hi; ++dd) {
          emit(c, dd, running);
          running = kNegInf;
        }
      }
    } else if (eg == 0 || two_groups) {
      // ---- rows mode: warp = one 32-row query chunk, all columns of the tile.
      for (int m = 0; m < g_this; ++m)
        if (!two_groups || (m & 1) == eg) carry[m * kQTileRows + row] = kNegInf;
      for (int64_t t0 = tok_lo; ok && t0 < tok_hi; t0 += TN) {
        int64_t next_doc = doc, next_dend = dend;
        for (int m = 0; m < g_this; ++m, ++u) {
          if (two_groups && (m & 1) != eg) continue;
          const uint32_t slot = u % NSLOT;
          if (!(ok = wait_full(slot, u))) break;
          tc_fence_after();
          const int chunk = (m_first + m) * 4 + lg;
          bool released = false;
          if (chunk < a.n_chunks_total) {
            float rm = carry[m * kQTileRows + row];
            int64_t dd = doc, de = dend;
            // Columns of this tile: [0, ncol) are tokens of the range; the open document ends
            // at column dcol (>= 0, clamped far past the tile when it ends later).
            const int ncol = (tok_hi - t0 < TN) ? static_cast<int>(tok_hi - t0) : TN;
            auto rel = [&](int64_t e) -> int {
              const int64_t x = e - t0;
              return x > 4 * TN ? 4 * TN : static_cast<int>(x);
            };
            int dcol = rel(de);
            const uint32_t tbase = t_lane + slot * TN;
            // 32 columns starting at column cb, all < ncol
            auto reduce32 = [&](const uint32_t(&v)[32], int cb) {
              if (dcol >= cb + 32 && ncol >= cb + 32) {
                rm = max32(rm, v);  // the whole block lies in the open document
                return;
              }
              if (QRES && ncol >= cb + 32) {
                // a full block whose only boundary is the open document's end (Q-resident
                // kernels only: compiled into the streaming kernel, the jump put the loaded block
                // in a 976-byte local-memory frame and made d = 256 / 768 scoring 2-5x slower)
                const int64_t de2 = doc_end(dd + 1);
                const int dcol2 = rel(de2);
                if (dcol2 >= cb + 32) {
                  const float next = split_max32(rm, v, dcol - cb);
                  emit(chunk, dd, rm);
                  rm = next;
                  ++dd;
                  de = de2;
                  dcol = dcol2;
                  return;
                }
              }
              {
                const int n = (ncol - cb < 32) ? ncol - cb : 32;
                int lo = 0;
                while (true) {
                  const int hi = (dcol - cb < n) ? dcol - cb : n;
                  rm = range_max32(rm, v, lo, hi);
                  if (dcol - cb >= n) break;
                  emit(chunk, dd, rm);
                  rm = kNegInf;
                  ++dd;
                  de = doc_end(dd);
                  dcol = rel(de);
                  lo = hi;
                }
              }
            };
            // TMEM loads double-buffered (block b+1 in flight while b is reduced): 64 columns
            // per load, 32 in the PQ variant (448 threads leave it fewer registers)
            // The slot goes back to the MMA as soon as its last block is in registers, before
            // that block is reduced: the reduction then overlaps the slot's refill.
            auto release_slot = [&]() {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(acce_bar(slot));
              released = true;
            };
            if constexpr (!PQ) {
              uint32_t ra[64], rb[64];
              tmem_ld64_async(tbase, ra);
#pragma unroll
              for (int b = 0; b < TN / 64; ++b) {
                uint32_t(&cur)[64] = (b & 1) ? rb : ra;
                uint32_t(&nxt)[64] = (b & 1) ? ra : rb;
                const int cb = 64 * b;
                if (cb < ncol) {
                  tmem_wait_ld(cur);
                  if (b + 1 < TN / 64 && cb + 64 < ncol) tmem_ld64_async(tbase + cb + 64, nxt);
                  else release_slot();
                  reduce32(*reinterpret_cast<const uint32_t(*)[32]>(&cur[0]), cb);
                  if (cb + 32 < ncol) reduce32(*reinterpret_cast<const uint32_t(*)[32]>(&cur[32]), cb + 32);
                }
              }
            } else {
              uint32_t ra[32], rb[32];
              tmem_ld32_async(tbase, ra);
#pragma unroll
              for (int b = 0; b < TN / 32; ++b) {
                uint32_t(&cur)[32] = (b & 1) ? rb : ra;
                uint32_t(&nxt)[32] = (b & 1) ? ra : rb;
                const int cb = 32 * b;
                if (cb < ncol) {
                  tmem_wait_ld32(cur);
                  if (b + 1 < TN / 32 && cb + 32 < ncol) tmem_ld32_async(tbase + cb + 32, nxt);
                  else release_slot();
                  reduce32(cur, cb);
                }
              }
            }
            carry[m * kQTileRows + row] = rm;
            next_doc = dd;
            next_dend = de;
          }
          if (!released) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acce_bar(slot));
          }
        }
        doc = next_doc;
        dend = next_dend;
      }
      if (ok) {
        // Documents still open at the end of the range: the last one (ends at tok_hi) and any
        // empty documents after it.
        for (int m = 0; m < g_this; ++m) {
          if (two_groups && (m & 1) != eg) continue;
          const int chunk = (m_first + m) * 4 + lg;
          if (chunk >= a.n_chunks_total) continue;
          float rm = carry[m * kQTileRows + row];
          for (int64_t dd = doc; dd < doc_hi; ++dd) {
            emit(chunk, dd, rm);
            rm = kNegInf;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// Packs Q (n_queries, nq, d) into 128-row M tiles: chunk c (32 rows) = rows [32p, 32p+32) of query
// c / nchunk (p = c % nchunk); rows past nq and chunks past the last query are zero. With
// `replicate` (one query tile of 1 or 2 chunks) quarter q of the tile holds chunk q % n_chunks.
__global__ void pack_query_tiles_kernel(const uint4* __restrict__ q, uint4* __restrict__ qp,
                                        int64_t n_vec_total, int vec_per_row, int nq, int nchunk,
                                        int n_chunks_total, int replicate) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n_vec_total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / vec_per_row;
    const int v = static_cast<int>(i - r * vec_per_row);
    // replicate: 1 or 2 chunks repeated over the tile's four 32-row quarters
    const int64_t c = replicate ? (r >> 5) % n_chunks_total : (r >> 5);
    const int ln = static_cast<int>(r & 31);
    uint4 val = make_uint4(0, 0, 0, 0);
    if (c < n_chunks_total) {
      const int64_t qi = c / nchunk;
      const int src = static_cast<int>(c - qi * nchunk) * 32 + ln;
      if (src < nq) val = q[(qi * nq + src) * vec_per_row + v];
    }
    qp[i] = val;
  }
}

// out[q, doc] = sum over the query's chunks, in chunk order (deterministic).
__global__ void sum_query_chunks_kernel(const float* __restrict__ partial, float* __restrict__ out,
                                        int64_t n_queries, int64_t n_docs, int nchunk) {
  const int64_t total = n_queries * n_docs;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t q = i / n_docs;
    const int64_t dd = i - q * n_docs;
    float s = 0.0f;
    for (int p = 0; p < nchunk; ++p) s += partial[(q * nchunk + p) * n_docs + dd];
    out[i] = s;
  }
}

__global__ void fill_kernel(float* out, int64_t n, float v) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = v;
}

struct DensePlan {
  int esize, cw, kc, nchunk, n_chunks_total, n_mtiles;
  int TN, G, stages, n_groups, n_ranges;
  bool qres;
  size_t qp_bytes, partial_bytes;
  uint32_t cb_bytes;
};

int plan_dense(int dtype, int64_t n_queries, int64_t nq, int64_t d, int64_t n_docs,
               int64_t n_tokens, int out_mode, int num_sms, int max_smem, DensePlan* p,
               uint32_t cb_bytes = 0, int prefer_tn = 0) {
  p->cb_bytes = cb_bytes;
  p->esize = (dtype == TMS_F32) ? 4 : 2;
  p->cw = 128 / p->esize;
  if ((d * p->esize) % 16 != 0) return TMS_ERR_UNSUPPORTED;
  p->kc = static_cast<int>((d + p->cw - 1) / p->cw);
  p->nchunk = static_cast<int>((nq + 31) / 32);
  const int64_t chunks = n_queries * p->nchunk;
  const int64_t mtiles = (chunks + 3) / 4;
  if (chunks > (int64_t(1) << 30) || mtiles * kQTileRows > (int64_t(1) << 31) - 1)
    return TMS_ERR_UNSUPPORTED;
  p->n_chunks_total = static_cast<int>(chunks);
  p->n_mtiles = static_cast<int>(mtiles);
  p->qp_bytes = align_up(static_cast<size_t>(mtiles) * kQTileRows * d * p->esize, 1024);
  p->partial_bytes = (out_mode == TMS_OUT_SCORE && p->nchunk > 1)
                         ? align_up(static_cast<size_t>(chunks) * n_docs * 4, 256)
                         : 0;

  // barriers, carries / exchange area, misc, and the PQ variant's codebook
  const int budget = max_smem - 2560 - 64 - static_cast<int>(align_up(cb_bytes, 16));
  // 256-token tiles at every width: an M=128 x N=256 MMA reads 12 KB of operands per 128 tensor
  // cycles (96 B/clk of the 128 B/clk shared-memory port), an N=128 one 8 KB per 64 cycles (the
  // whole port), and for d > 128 the TMA writes of the streamed chunks share the same port
  // (measured at 16 queries x 50k x 256 tokens: d=768 9.7 ms vs 12.2 ms with 128-token tiles,
  // d=256 3.1 vs 3.3 ms). The cost is two TMEM accumulator slots instead of four.
  p->TN = prefer_tn ? prefer_tn : 256;
  if (p->TN != 128 && p->TN != 256) p->TN = 256;
  const int stage_d = p->kc * p->TN * 128;
  const int qtile = p->kc * static_cast<int>(kQChunkBytes);
  p->qres = qtile + 2 * stage_d <= budget;
  if (cb_bytes && !p->qres) return TMS_ERR_UNSUPPORTED;  // the PQ variant keeps Q resident
  if (p->qres) {
    int gmax = (budget - 2 * stage_d) / qtile;
    gmax = gmax < 4 ? gmax : 4;
    if (gmax < 1) gmax = 1;
    // Per-CTA time grows with G x ceil(n_mtiles / G) (units per tile x token share), and an odd
    // G (> 0) runs the epilogue on one warp group instead of two: take the group size that
    // minimises the cost, the larger one on ties (fewer re-reads of each doc tile).
    int g = 1;
    int64_t best = 2 * static_cast<int64_t>(p->n_mtiles);
    for (int c = 2; c <= gmax && c <= p->n_mtiles; ++c) {
      const int64_t cost = static_cast<int64_t>(c) * ((p->n_mtiles + c - 1) / c) * ((c & 1) ? 2 : 1);
      if (cost <= best) { best = cost; g = c; }
    }
    p->n_groups = (p->n_mtiles + g - 1) / g;
    p->G = (p->n_mtiles + p->n_groups - 1) / p->n_groups;
    int st = (budget - p->G * qtile) / stage_d;
    st = st > 4 ? 4 : st;
    p->stages = st;
  } else {
    const int stage = static_cast<int>(kQChunkBytes) + p->TN * 128;
    int g = p->n_mtiles < 4 ? p->n_mtiles : 4;
    p->n_groups = (p->n_mtiles + g - 1) / g;
    p->G = (p->n_mtiles + p->n_groups - 1) / p->n_groups;
    int st = budget / stage;
    st = st > 6 ? 6 : st;
    p->stages = st;
  }
  if (p->stages < 1) p->stages = 1;
  const bool split = p->n_mtiles == 1;
  // the estimate above reserved a fixed allowance for barriers / carries / exchange area: move
  // the stage count to what the exact layout allows (at most 4)
  {
    while (p->stages > 1 && static_cast<int>(dense_smem_layout(p->TN, p->qres, p->G, p->kc, p->stages,
                                                               split, p->cb_bytes).total) > max_smem)
      --p->stages;
    while (p->stages < 4 && static_cast<int>(dense_smem_layout(p->TN, p->qres, p->G, p->kc, p->stages + 1,
                                                               split, p->cb_bytes).total) <= max_smem)
      ++p->stages;
  }
  const SmemLayout L = dense_smem_layout(p->TN, p->qres, p->G, p->kc, p->stages, split, p->cb_bytes);
  if (static_cast<int>(L.total) > max_smem) return TMS_ERR_UNSUPPORTED;
  // Token ranges per query group: the fewest that make groups x ranges a multiple of the SM count
  // (one balanced wave or several), but never fewer than fill one wave.
  int64_t gcd = num_sms, gb = p->n_groups;
  while (gb) { const int64_t t = gcd % gb; gcd = gb; gb = t; }
  int64_t ranges = num_sms / gcd;
  if (p->n_groups < num_sms && ranges < num_sms / p->n_groups) ranges = num_sms / p->n_groups;
  const int64_t tiles = (n_tokens + p->TN - 1) / p->TN;
  if (ranges > tiles) ranges = tiles;
  if (ranges > n_docs) ranges = n_docs;
  if (ranges < 1) ranges = 1;
  p->n_ranges = static_cast<int>(ranges);
  if (static_cast<int64_t>(p->n_ranges) * p->n_groups > 0x7fffffffLL) return TMS_ERR_UNSUPPORTED;
  return TMS_OK;
}

template <int TN, bool QRES, bool TF32, bool PQ = false, int RES = 0>
int launch_dense_t(const CUtensorMap& qm, const CUtensorMap& dm, const DenseArgs& args,
                   const DensePlan& p, cudaStream_t st) {
  auto kern = dense_maxsim_kernel<TN, QRES, TF32, PQ, RES>;
  const SmemLayout L = dense_smem_layout(TN, QRES, p.G, p.kc, p.stages, p.n_mtiles == 1,
                                         p.cb_bytes);
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total);
  if (e != cudaSuccess) return TMS_ERR_CUDA;
  const unsigned grid = static_cast<unsigned>(p.n_ranges) * static_cast<unsigned>(p.n_groups);
  kern<<<grid, RES ? res_threads(RES) : PQ ? kPqThreadsMma : kThreads, L.total, st>>>(qm, dm, args);
  return cuda_status(cudaGetLastError());
}

int launch_dense(const CUtensorMap& qm, const CUtensorMap& dm, const DenseArgs& args,
                 const DensePlan& p, bool tf32, cudaStream_t st) {
  if (tf32) {
    if (p.TN == 256)
      return p.qres ? launch_dense_t<256, true, true>(qm, dm, args, p, st)
                    : launch_dense_t<256, false, true>(qm, dm, args, p, st);
    return p.qres ? launch_dense_t<128, true, true>(qm, dm, args, p, st)
                  : launch_dense_t<128, false, true>(qm, dm, args, p, st);
  }
  if (p.TN == 256)
    return p.qres ? launch_dense_t<256, true, false>(qm, dm, args, p, st)
                  : launch_dense_t<256, false, false>(qm, dm, args, p, st);
  return p.qres ? launch_dense_t<128, true, false>(qm, dm, args, p, st)
                : launch_dense_t<128, false, false>(qm, dm, args, p, st);
}

}  // namespace

}  // namespace tms

using namespace tms;

extern "C" size_t tms_dense_workspace_size(int dtype, int64_t n_queries, int64_t nq, int64_t d,
                                           int64_t n_docs, int out_mode) {
  if (n_queries <= 0 || nq <= 0 || d <= 0 || n_docs < 0) return 0;
  DensePlan p;
  if (plan_dense(dtype, n_queries, nq, d, n_docs, 1, out_mode, 148, 232448, &p) != TMS_OK)
    return 0;
  return p.qp_bytes + p.partial_bytes;
}

extern "C" int tms_dense_maxsim(const void* Q, int dtype, int64_t n_queries, int64_t nq,
                                int64_t d, const void* D, int64_t n_tokens,
                                const int64_t* doc_offsets, int64_t n_docs, int64_t nd_uniform,
                                float* out, int out_mode, void* workspace,
                                size_t workspace_bytes, void* stream) {
  NvtxRange nvtx_range("tms_dense_maxsim");
  if (dtype != TMS_F16 && dtype != TMS_BF16 && dtype != TMS_F32) return TMS_ERR_INVALID;
  if (out_mode != TMS_OUT_SCORE && out_mode != TMS_OUT_TOKEN_MAX) return TMS_ERR_INVALID;
  if (n_queries < 0 || nq < 0 || d <= 0 || n_docs < 0 || n_tokens < 0) return TMS_ERR_INVALID;
  if (n_queries == 0 || n_docs == 0) return TMS_OK;
  if (nq == 0) return TMS_ERR_INVALID;
  if (!Q || !out || (n_tokens > 0 && !D)) return TMS_ERR_INVALID;
  if (!doc_offsets && nd_uniform < 0) return TMS_ERR_INVALID;
  if (n_tokens >= (int64_t(1) << 31)) return TMS_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(Q) & 15) || (reinterpret_cast<uintptr_t>(D) & 15))
    return TMS_ERR_INVALID;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int status = TMS_OK;
  const DeviceInfo* dev = current_device_info(&status);
  if (!dev) return status;

  const int64_t out_elems = (out_mode == TMS_OUT_SCORE) ? n_queries * n_docs : n_queries * n_docs * nq;
  if (n_tokens == 0 || (!doc_offsets && nd_uniform == 0)) {
    // No token at all: every document is empty and scores -inf.
    fill_kernel<<<dev->num_sms * 4, 256, 0, st>>>(out, out_elems, -__builtin_huge_valf());
    return cuda_status(cudaGetLastError());
  }
  if (!doc_offsets && n_docs * nd_uniform > n_tokens) return TMS_ERR_INVALID;

  DensePlan p;
  int rc = plan_dense(dtype, n_queries, nq, d, n_docs, n_tokens, out_mode, dev->num_sms,
                      dev->max_smem_optin, &p);
  if (rc != TMS_OK) return rc;
  if (!workspace || workspace_bytes < p.qp_bytes + p.partial_bytes) return TMS_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 1023) return TMS_ERR_INVALID;

  uint8_t* qp = static_cast<uint8_t*>(workspace);
  float* partial = reinterpret_cast<float*>(qp + p.qp_bytes);
  const int row_bytes = static_cast<int>(d * p.esize);
  const int vpr = row_bytes / 16;
  const int64_t n_vec = static_cast<int64_t>(p.n_mtiles) * kQTileRows * vpr;
  {
    int blocks = static_cast<int>((n_vec + 255) / 256);
    if (blocks > dev->num_sms * 8) blocks = dev->num_sms * 8;
    pack_query_tiles_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint4*>(Q),
                                                    reinterpret_cast<uint4*>(qp), n_vec, vpr,
                                                    static_cast<int>(nq), p.nchunk,
                                                    p.n_chunks_total, p.n_mtiles == 1 && p.n_chunks_total <= 2);
    if (cudaGetLastError() != cudaSuccess) return TMS_ERR_CUDA;
  }

  const CUtensorMapDataType dt = (dtype == TMS_F16)    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                 : (dtype == TMS_BF16) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUtensorMap qm, dm;
  rc = encode_tmap_2d(&qm, dt, qp, static_cast<uint64_t>(d),
                      static_cast<uint64_t>(p.n_mtiles) * kQTileRows, row_bytes, p.cw, kQTileRows);
  if (rc != TMS_OK) return rc;
  rc = encode_tmap_2d(&dm, dt, D, static_cast<uint64_t>(d), static_cast<uint64_t>(n_tokens),
                      row_bytes, p.cw, p.TN);
  if (rc != TMS_OK) return rc;

  DenseArgs args;
  args.docs.offsets = doc_offsets;
  args.docs.n_docs = n_docs;
  args.docs.nd = doc_offsets ? 0 : nd_uniform;
  args.out = (out_mode == TMS_OUT_SCORE && p.nchunk > 1) ? partial : out;
  args.err = dev->err_word;
  args.timeout_ns = wait_timeout_ns();
  args.n_chunks_total = p.n_chunks_total;
  args.nchunk = p.nchunk;
  args.nq = static_cast<int>(nq);
  args.n_mtiles = p.n_mtiles;
  args.G = p.G;
  args.n_groups = p.n_groups;
  args.n_ranges = p.n_ranges;
  args.kc = p.kc;
  args.stages = p.stages;
  args.out_mode = out_mode;
  args.ab_format = (dtype == TMS_F16) ? 0u : (dtype == TMS_BF16) ? 1u : 2u;
  args.codes = nullptr;
  args.n_code_rows = 0;
  args.codebook = nullptr;
  args.cb_dtype = args.pq_M = args.pq_K = args.pq_dsub = 0;
  args.cb_bytes = 0;
  args.debug_flags = debug_flags();

  rc = launch_dense(qm, dm, args, p, dtype == TMS_F32, st);
  if (rc != TMS_OK) return rc;
  if (out_mode == TMS_OUT_SCORE && p.nchunk > 1) {
    const int64_t total = n_queries * n_docs;
    int blocks = static_cast<int>((total + 255) / 256);
    if (blocks > dev->num_sms * 8) blocks = dev->num_sms * 8;
    sum_query_chunks_kernel<<<blocks, 256, 0, st>>>(partial, out, n_queries, n_docs, p.nchunk);
    return cuda_status(cudaGetLastError());
  }
  return TMS_OK;
}

// Exposes the launch plan for tests and the benchmark (not part of the stable ABI).
extern "C" int tms_dense_plan_info(int dtype, int64_t n_queries, int64_t nq, int64_t d,
                                   int64_t n_docs, int64_t n_tokens, int out_mode, int num_sms,
                                   int64_t* info /* 10 entries */) {
  DensePlan p;
  int rc = plan_dense(dtype, n_queries, nq, d, n_docs, n_tokens, out_mode, num_sms, 232448, &p);
  if (rc != TMS_OK) return rc;
  info[0] = p.TN;
  info[1] = p.qres;
  info[2] = p.G;
  info[3] = p.stages;
  info[4] = p.n_groups;
  info[5] = p.n_ranges;
  info[6] = p.n_mtiles;
  info[7] = p.kc;
  info[8] = dense_smem_layout(p.TN, p.qres, p.G, p.kc, p.stages, p.n_mtiles == 1, 0).total;
  info[9] = static_cast<int64_t>(p.n_ranges) * p.n_groups;
  return TMS_OK;
}

// ------------------------------------------------------------------------------------------------
// PQ-ADC on the tensor cores: the dense kernel with decoder warps (see the kernel's PQ branch).
// ------------------------------------------------------------------------------------------------
namespace tms {

// fp16 codebook bytes if the tensor-core PQ path can take this shape, else 0.
size_t pq_mma_codebook_bytes(int64_t M, int64_t K, int64_t dsub) {
  const int64_t d = M * dsub;
  if (K < 1 || K > 256 || dsub % 8 != 0 || d % 64 != 0 || d > 512) return 0;
  const int64_t b = M * K * dsub * 2;
  return b <= 96 * 1024 ? static_cast<size_t>(b) : 0;
}

size_t pq_mma_workspace_size(int64_t n_queries, int64_t nq, int64_t d, int64_t n_docs) {
  return tms_dense_workspace_size(TMS_F16, n_queries, nq, d, n_docs, TMS_OUT_SCORE);
}

// The dense kernel with decoder warps (PQ codes or residual-compressed tokens): query packing,
// the Q tensor map, the launch, and the chunk sum for Nq > 32. `fill` sets the decoder's fields
// of the argument block.
template <bool RES, typename Fill>
int decoder_maxsim(const void* Q, int64_t n_queries, int64_t nq, int64_t d, uint32_t cb_bytes,
                   int64_t n_tokens, const int64_t* doc_offsets, int64_t n_docs, int64_t nd_uniform,
                   float* out, void* workspace, size_t workspace_bytes, cudaStream_t st, Fill fill) {
  if (n_tokens <= 0 || n_tokens >= (int64_t(1) << 31)) return TMS_ERR_UNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(Q) & 15) return TMS_ERR_UNSUPPORTED;
  int status = TMS_OK;
  const DeviceInfo* dev = current_device_info(&status);
  if (!dev) return status;
  DensePlan p;
  int rc = plan_dense(TMS_F16, n_queries, nq, d, n_docs, n_tokens, TMS_OUT_SCORE, dev->num_sms,
                      dev->max_smem_optin, &p, cb_bytes,
                      /* 128-token tiles: two query tiles per CTA fit beside the codebook */ 128);
  if (rc != TMS_OK) return rc;
  if (RES && p.TN != 128) return TMS_ERR_UNSUPPORTED;  // the residual decoders fill 128-token tiles
  if (!workspace || workspace_bytes < p.qp_bytes + p.partial_bytes) return TMS_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 1023) return TMS_ERR_INVALID;
  uint8_t* qp = static_cast<uint8_t*>(workspace);
  float* partial = reinterpret_cast<float*>(qp + p.qp_bytes);
  const int row_bytes = static_cast<int>(d * 2);
  const int vpr = row_bytes / 16;
  const int64_t n_vec = static_cast<int64_t>(p.n_mtiles) * kQTileRows * vpr;
  int blocks = static_cast<int>((n_vec + 255) / 256);
  if (blocks > dev->num_sms * 8) blocks = dev->num_sms * 8;
  pack_query_tiles_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint4*>(Q),
                                                  reinterpret_cast<uint4*>(qp), n_vec, vpr,
                                                  static_cast<int>(nq), p.nchunk, p.n_chunks_total,
                                                  p.n_mtiles == 1 && p.n_chunks_total <= 2);
  if (cudaGetLastError() != cudaSuccess) return TMS_ERR_CUDA;
  CUtensorMap qm;
  rc = encode_tmap_2d(&qm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, qp, static_cast<uint64_t>(d),
                      static_cast<uint64_t>(p.n_mtiles) * kQTileRows, row_bytes, p.cw, kQTileRows);
  if (rc != TMS_OK) return rc;
  DenseArgs args = {};
  args.docs.offsets = doc_offsets;
  args.docs.n_docs = n_docs;
  args.docs.nd = doc_offsets ? 0 : nd_uniform;
  args.out = p.nchunk > 1 ? partial : out;
  args.err = dev->err_word;
  args.timeout_ns = wait_timeout_ns();
  args.n_chunks_total = p.n_chunks_total;
  args.nchunk = p.nchunk;
  args.nq = static_cast<int>(nq);
  args.n_mtiles = p.n_mtiles;
  args.G = p.G;
  args.n_groups = p.n_groups;
  args.n_ranges = p.n_ranges;
  args.kc = p.kc;
  args.stages = p.stages;
  args.out_mode = TMS_OUT_SCORE;
  args.ab_format = 0u;
  args.n_code_rows = n_tokens;
  args.cb_bytes = cb_bytes;
  args.debug_flags = debug_flags();
  fill(args);
  if constexpr (RES) {
    // eight decoder warps (two per scheduler): the decoding is latency-bound, and the second warp
    // per scheduler is worth more than the registers it costs (96 per thread at 576 threads, with
    // a few spills): 18.2 ms against 23.2 ms with four warps at 128 registers (1 query, 1M x 128
    // tokens, nbits = 2)
    rc = launch_dense_t<128, true, false, true, kResDecWarps>(qm, qm, args, p, st);
  } else if (p.TN == 256) {
    rc = launch_dense_t<256, true, false, true, 0>(qm, qm, args, p, st);
  } else {
    rc = launch_dense_t<128, true, false, true, 0>(qm, qm, args, p, st);
  }
  if (rc != TMS_OK || p.nchunk == 1) return rc;
  const int64_t total = n_queries * n_docs;
  blocks = static_cast<int>((total + 255) / 256);
  if (blocks > dev->num_sms * 8) blocks = dev->num_sms * 8;
  sum_query_chunks_kernel<<<blocks, 256, 0, st>>>(partial, out, n_queries, n_docs, p.nchunk);
  return cuda_status(cudaGetLastError());
}

int pq_mma_maxsim(const void* Q, int64_t n_queries, int64_t nq, const void* codebook, int cb_dtype,
                  int64_t M, int64_t K, int64_t dsub, const uint8_t* codes, int64_t n_tokens,
                  const int64_t* doc_offsets, int64_t n_docs, int64_t nd_uniform, float* out,
                  void* workspace, size_t workspace_bytes, cudaStream_t st) {
  const size_t cb_bytes = pq_mma_codebook_bytes(M, K, dsub);
  if (!cb_bytes) return TMS_ERR_UNSUPPORTED;
  return decoder_maxsim<false>(Q, n_queries, nq, M * dsub, static_cast<uint32_t>(cb_bytes), n_tokens,
                               doc_offsets, n_docs, nd_uniform, out, workspace, workspace_bytes, st,
                               [&](DenseArgs& a) {
                                 a.codes = codes;
                                 a.codebook = codebook;
                                 a.cb_dtype = cb_dtype;
                                 a.pq_M = static_cast<int>(M);
                                 a.pq_K = static_cast<int>(K);
                                 a.pq_dsub = static_cast<int>(dsub);
                               });
}

}  // namespace tms

// ------------------------------------------------------------------------------------------------
// No-allocation variant of tms_dense_maxsim.
//
// Some callers cannot give this library device memory: a serving engine that reserves all of the
// GPU's memory for its own pool at start-up and forbids other allocations, or a host plug-in that
// must never call cudaMalloc (it can synchronise the whole device and fail under memory pressure)
// and has no allocator of its own to pass in. For them the dense kernel's scratch -- the packed
// query tiles and, for queries longer than 32 tokens, the per-chunk partial sums -- lives in the
// fixed array below instead of a caller workspace. Every GPU that loads the library holds the
// array until the process exits.
// ------------------------------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // usable scratch: 4 MiB per device
constexpr size_t kNoAllocAlign = 1024;                     // the workspace alignment tms_dense_maxsim wants
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes + kNoAllocAlign];

std::mutex g_noalloc_mutex;
struct NoAllocBase {
  void* ctx;      // context the address was looked up in
  uint8_t* base;  // device address of the array, 1024-aligned
};
NoAllocBase g_noalloc_base[64] = {};

// Host code must not use the array's name as a device address: look the address up with the
// device current and cache it per device and context (a new context, e.g. after cudaDeviceReset,
// loads the module again at another address, so the lookup is repeated there).
int noalloc_scratch(uint8_t** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return TMS_ERR_CUDA;
  void* ctx = current_cu_context();
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  NoAllocBase& b = g_noalloc_base[dev];
  if (!b.base || b.ctx != ctx) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return TMS_ERR_CUDA;
    const uintptr_t a = (reinterpret_cast<uintptr_t>(p) + kNoAllocAlign - 1) & ~(kNoAllocAlign - 1);
    b.base = reinterpret_cast<uint8_t*>(a);
    b.ctx = current_cu_context();  // cudaGetSymbolAddress may have made the primary context current
  }
  *out = b.base;
  return TMS_OK;
}

}  // namespace

extern "C" int tms_dense_maxsim_noalloc(const void* Q, int dtype, int64_t n_queries, int64_t nq,
                                        int64_t d, const void* D, int64_t n_tokens,
                                        const int64_t* doc_offsets, int64_t n_docs,
                                        int64_t nd_uniform, float* out, int out_mode,
                                        void* stream) {
  NvtxRange nvtx_range("tms_dense_maxsim_noalloc");
  // Nothing in the scratch has to start at zero: the pack kernel writes every byte of the query
  // tiles (padding included) and every partial sum is written before it is read.
  // The scratch size depends only on the problem (packed query tiles and per-chunk partial sums),
  // not on the device: tms_dense_workspace_size plans with fixed device facts, and the check
  // below on the inner call's answer covers any future dependence on the real device.
  const size_t need = tms_dense_workspace_size(dtype, n_queries, nq, d, n_docs, out_mode);
  if (need > kNoAllocScratchBytes) return TMS_ERR_TOO_LARGE;
  uint8_t* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc != TMS_OK) return rc;
  rc = tms_dense_maxsim(Q, dtype, n_queries, nq, d, D, n_tokens, doc_offsets, n_docs, nd_uniform,
                        out, out_mode, scratch, kNoAllocScratchBytes, stream);
  return rc == TMS_ERR_WORKSPACE ? TMS_ERR_TOO_LARGE : rc;
}

// ------------------------------------------------------------------------------------------------
// Residual-compressed corpora: token = centroids[code] + bucket_weights[per-dimension index]
// (optionally L2-normalised), decoded on chip by the dense kernel's decoder warps.
// ------------------------------------------------------------------------------------------------
extern "C" size_t tms_residual_workspace_size(int64_t n_queries, int64_t nq, int64_t d,
                                              int64_t n_docs) {
  if (n_queries <= 0 || nq <= 0 || d <= 0 || d > 128 || d % 64 != 0 || n_docs < 0) return 0;
  const size_t dense = tms_dense_workspace_size(TMS_F16, n_queries, nq, d, n_docs, TMS_OUT_SCORE);
  const size_t rows = tms::pq_tokrows_workspace_size(n_queries, nq, n_docs);  // token-rows kernel
  return dense > rows ? dense : rows;
}

extern "C" int tms_residual_maxsim(const void* Q, int64_t n_queries, int64_t nq, int64_t d,
                                   const void* centroids, int64_t n_centroids, const int32_t* codes,
                                   const uint8_t* residuals, const float* bucket_weights, int nbits,
                                   int normalize, int64_t n_tokens, const int64_t* doc_offsets,
                                   int64_t n_docs, int64_t nd_uniform, float* out, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  tms::NvtxRange nvtx_range("tms_residual_maxsim");
  if (n_queries < 0 || nq <= 0 || d <= 0 || n_docs < 0 || n_tokens < 0 || n_centroids < 1)
    return TMS_ERR_INVALID;
  if (nbits != 1 && nbits != 2 && nbits != 4) return TMS_ERR_INVALID;
  if (d % 64 != 0 || d > 128) return TMS_ERR_UNSUPPORTED;
  if (n_queries == 0 || n_docs == 0) return TMS_OK;
  if (!Q || !centroids || !bucket_weights || !out || (n_tokens > 0 && (!codes || !residuals)))
    return TMS_ERR_INVALID;
  if (!doc_offsets && (nd_uniform < 0 || n_docs * nd_uniform > n_tokens)) return TMS_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(centroids) & 15) || (reinterpret_cast<uintptr_t>(residuals) & 3) ||
      (reinterpret_cast<uintptr_t>(codes) & 3))
    return TMS_ERR_INVALID;  // 16-byte centroid rows, 32-bit residual words and codes
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n_tokens == 0) {  // every document is empty
    int status = TMS_OK;
    const tms::DeviceInfo* dev = tms::current_device_info(&status);
    if (!dev) return status;
    const int64_t total = n_queries * n_docs;
    int blocks = static_cast<int>((total + 255) / 256);
    if (blocks > dev->num_sms * 8) blocks = dev->num_sms * 8;
    tms::fill_kernel<<<blocks, 256, 0, st>>>(out, total, tms::kNegInf);
    return tms::cuda_status(cudaGetLastError());
  }
  // up to four 32-row query chunks: the token-rows kernel (decoded tokens as the TMEM A operand,
  // one document stream per lane); larger batches: the dense kernel's residual decoder warps
  if (((nq + 31) / 32) * n_queries <= 4) {
    const int rc = tms::res_tokrows_maxsim(Q, n_queries, nq, d, centroids, n_centroids, codes,
                                           residuals, bucket_weights, nbits, normalize, n_tokens,
                                           doc_offsets, n_docs, nd_uniform, out, workspace,
                                           workspace_bytes, st);
    if (rc != TMS_ERR_UNSUPPORTED) return rc;
  }
  return tms::decoder_maxsim<true>(
      Q, n_queries, nq, d, tms::residual_layout(static_cast<int>(d), nbits).total, n_tokens, doc_offsets, n_docs,
      nd_uniform, out, workspace, workspace_bytes, st, [&](tms::DenseArgs& a) {
        a.res_centroids = static_cast<const __half*>(centroids);
        a.res_codes = codes;
        a.res_bits = residuals;
        a.res_bw = bucket_weights;
        a.res_ncent = n_centroids;
        a.res_nbits = nbits;
        a.res_normalize = normalize ? 1 : 0;
      });
}
