// pq_tokrows.cu -- PQ-ADC and residual-compressed (ColBERTv2) corpora on the sm_100a tensor
// cores for small query batches (up to four 32-row query chunks), with the document tokens on the
// TMEM lanes.
//
//   score[q, doc] = sum_i max_{j in doc} sum_m <Q[q,i,m*dsub:(m+1)*dsub], C[m, codes[j,m], :]>
//
// Reference semantics: src/flash_pqsim_kernel.py:190-211 (distance table T[i,m,k] = <q_i,m, c_m,k>)
// and :213-280 (TileMaxSimPQ.score_batch: per token the sum over subspaces of T[i,m,code_m], max
// over the document's tokens, sum over the query tokens). The sum over m of <q_i,m, c_m,code_m>
// is <q_i, decode(codes_j)>, the dot product with the token's reconstructed vector, so the kernel
// rebuilds each token from the codebook and lets the tensor cores take the dot products.
//
// Design (the single-query PQ hot path):
//  * Decoded tokens are the MMA's A operand: M = 128 token rows x K = d, written from registers
//    straight into TMEM with tcgen05.st (lane = token, 32-bit column c = fp16 elements 2c, 2c+1).
//    No shared-memory store and no replicated query tile: the shared-memory traffic per token is
//    the codebook gather (M random 16-byte reads at dsub = 8). What paces the kernel is the MMA
//    reading its A operand from TMEM beside the decoders' stores and the epilogue's loads.
//    Residual corpora (modes kTrRes*): the decoders rebuild tokens from a centroid row and the
//    residual bits instead of codebook rows; the rest of the kernel is shared.
//  * The query rows are the B operand (N = 32, 64 or 128), resident in shared memory in the 128-byte-
//    swizzle K-major layout. S^T = Dtile . Q^T lands with one token per TMEM lane and one query row
//    per column.
//  * The CTA's token range (cut at document boundaries) is cut again into four document-aligned
//    sub-ranges, one per TMEM lane quarter, and each lane of a quarter walks its own documents:
//    lane l takes the quarter's documents l, l + 32, l + 64, ..., one token per tile, so TMEM lane
//    32q + l of tile j holds the j-th token of lane l's document stream (LaneDocs). A document
//    therefore lives on one lane: no cross-lane reduction, deterministic results.
//  * Epilogue: lane l keeps the running max over its document's tokens for every query row
//    (elementwise, registers); when the document ends, the lane sums its row maxima and stores
//    the score -- no shuffles (they share the shared-memory pipe that the decoders' codebook
//    gathers fill) and no walk over document boundaries inside a tile.
//  * A hand-off through an mbarrier costs ~500 cycles on this part, so TMEM holds as many tiles
//    in flight as fit (5 at N = 32: 64 decoded-token columns + 32 accumulator columns each).
//
// Warp roles (one or two chunks, 512 threads): warp 1 = TMEM owner + MMA issuer; warps 4..11 =
// decoders (lane quarter = warp % 4; the quarter's two warps rebuild alternate 64-element column
// blocks of every tile); warps 12..15 = epilogue (lane quarter = warp % 4); warps 0, 2, 3 only
// help in the prologue. Three or four chunks: warps 0..3 are a second epilogue group and the
// last decoder warp to finish a tile issues its MMAs (TrShape).
#include <cuda/atomic>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "tms_device.cuh"
#include "tms_internal.h"

namespace tms {

namespace {

constexpr int kTrThreads = 512;
constexpr int kTrDecWarp0 = 4;
constexpr int kTrEpiWarp0 = 12;
constexpr int kTrMaxChunks = 4;  // N = 32 x chunks <= 128 query rows per CTA (3 run as 4)
constexpr float kTrNegInf = -__builtin_huge_valf();

struct TrArgs {
  DocLayout docs;
  const uint8_t* codes;
  int64_t n_tokens;  // rows of codes: the quarters' token ranges are clamped to [0, n_tokens)
  const __half* Q;  // (n_queries, nq, d) fp16
  const void* codebook;
  float* out;  // (n_chunks, n_docs): final scores when nchunk == 1, else per-chunk partials
  uint32_t* err;
  uint64_t timeout_ns;
  int cb_dtype, M, K, dsub, d;
  int nq, nchunk, n_chunks;  // query rows per query, 32-row chunks per query, chunks in total
  int nslot;                 // TMEM slots (A columns + accumulator columns each)
  int n_ranges;
  int debug_flags;  // bit 0: decoders write nothing (exercises the bounded waits)
  // residual-compressed corpora (modes kTrRes1/2/4): token t = centroids[rcodes[t]] + bucket
  // weights of its residual row (rbytes bytes), scaled to unit length when normalize != 0
  const __half* cent;
  int64_t ncent;
  const int32_t* rcodes;
  const uint8_t* rbits;
  const float* bucket_w;
  int rbytes, normalize;
};

// Decoder modes (kernel template parameter): PQ with an fp16 codebook, PQ with the codebook split
// into fp16 hi + lo, residual codes with 1, 2 or 4 bits per dimension.
constexpr int kTrPq = 0, kTrPqSplit = 1, kTrRes1 = 2, kTrRes2 = 3, kTrRes4 = 4;
// Residual mode: a 16-entry table of bucket weights per 4 residual bits (4 / nbits dimensions an
// entry), the decoders' partial sums of squares per (slot, lane quarter, half, lane), and each
// decoder warp's ring of kTrResRing tiles: per lane its token's centroid half-row (pitch
// d + 16 bytes) and residual half-row (pitch tr_res_pb: conflict-free vector reads).
constexpr int kTrResRing = 3;
__host__ __device__ inline int tr_res_pb(int rw) { return rw == 8 ? 48 : 4 * rw; }
__host__ __device__ inline uint32_t tr_res_slot(int d, int nb) {
  return 32u * static_cast<uint32_t>(d + 16 + tr_res_pb(d / 2 * nb / 32));
}
__host__ __device__ inline uint32_t tr_res_bytes(int nslot, int d, int nb) {
  return 256u + static_cast<uint32_t>(nslot) * 4u * 2u * 32u * 4u + 8u * kTrResRing * tr_res_slot(d, nb);
}

struct TrLayout {
  uint32_t b_off, cb_off, bar_off, misc_off, total;
};
__host__ __device__ inline TrLayout tr_layout(int N, int d, uint32_t cb_bytes, int nslot) {
  TrLayout L;
  L.b_off = 0;
  L.cb_off = static_cast<uint32_t>((d / 64) * N * 128);
  L.bar_off = (L.cb_off + cb_bytes + 15u) & ~15u;
  L.misc_off = L.bar_off + static_cast<uint32_t>(3 * nslot + 1) * 8u;
  L.total = L.misc_off + 128u;
  return L;
}
struct TrMisc {
  uint32_t tmem;
  int abort;
  int never;  // stays 0: the final drain wait is bounded by time only
  int n_tiles;
  int64_t sub_doc[5];
  uint32_t arrivals[8];  // decoder warps done with the slot's tiles (the last one issues the MMAs)
};

template <bool kPos>  // kPos: track token positions (decoders); the epilogue needs counts only
struct LaneDocs {
  int64_t first;  // the quarter's first document (absolute)
  int ndq;        // documents in the quarter
  int d;          // current document (relative); >= ndq once the lane is done
  int rem;        // tokens of d not yet handed out (> 0 while the lane is active)
  int n_len;      // length of document d + 32, fetched one document ahead
  int64_t pos;    // absolute index of the lane's next token (kPos)
  int64_t n_start;  // start of document d + 32 (kPos)

  __device__ __forceinline__ bool active() const { return d < ndq; }
  // length (clamped to [0, 2^31)) and start of relative document dd; (0, 0) past the quarter
  __device__ __forceinline__ int fetch(const DocLayout& docs, int dd, int64_t& st) const {
    st = 0;
    if (dd >= ndq) return 0;
    st = docs.start(first + dd);
    const int64_t e = docs.start(first + dd + 1) - st;
    return e < 0 ? 0 : (e > 0x7fffffffLL ? 0x7fffffff : static_cast<int>(e));
  }
  __device__ __forceinline__ void advance(const DocLayout& docs) {
    d += 32;
    rem = n_len;
    int64_t st;
    if (kPos) pos = n_start;
    n_len = fetch(docs, d + 32, st);
    if (kPos) n_start = st;
  }
  // Move to the next non-empty document; on_empty(dd) for every empty one passed over.
  template <class F>
  __device__ __forceinline__ void next(const DocLayout& docs, F&& on_empty) {
    advance(docs);
    while (rem == 0 && d < ndq) {
      on_empty(d);
      advance(docs);
    }
  }
  template <class F>
  __device__ __forceinline__ void init(const DocLayout& docs, int64_t first_, int ndq_, int lane, F&& on_empty) {
    first = first_;
    ndq = ndq_;
    d = lane - 32;
    int64_t st;
    n_len = fetch(docs, lane, st);
    n_start = st;
    pos = 0;
    next(docs, on_empty);
  }
  // After the lane's token of a tile: on_done(d) when that was the document's last token.
  template <class G, class F>
  __device__ __forceinline__ void step(const DocLayout& docs, G&& on_done, F&& on_empty) {
    if (d < ndq) {
      if (kPos) ++pos;
      if (--rem == 0) {
        on_done(d);
        next(docs, on_empty);
      }
    }
  }
};

// Last-arriver hand-off: a decoder warp's lane 0 counts its finished tile into the slot's counter
// (acq_rel, after tcgen05.fence::before_thread_sync); the eighth arrival sees every decoder's
// TMEM stores and issues the MMAs itself, so no thread waits for the slowest decoder.
// The counter only grows (the k-th use of a slot counts 8k .. 8k + 7; wrap-around keeps that).
__device__ __forceinline__ uint32_t count_arrival(uint32_t* ctr) {
  cuda::atomic_ref<uint32_t, cuda::thread_scope_block> ref(*ctr);
  return ref.fetch_add(1, cuda::memory_order_acq_rel);
}

template <int NCH> struct TrShape {
  static constexpr bool kMmaInDecoder = NCH > 2;
  static constexpr int kTmemWarp = NCH > 2 ? kTrDecWarp0 : 1;
  static constexpr int kEpiWarps = NCH > 2 ? 8 : 4;
  static constexpr int kEpiChunks = NCH > 2 ? NCH / 2 : NCH;  // chunks per epilogue warp
};

template <int NCH, int MODE>
__global__ void __launch_bounds__(kTrThreads, 1) pq_tokrows_kernel(const TrArgs a) {
  using Shape = TrShape<NCH>;
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int N = NCH * 32;
  constexpr bool SPLIT = MODE == kTrPqSplit;
  constexpr bool RES = MODE >= kTrRes1;
  constexpr int NB = RES ? (1 << (MODE - kTrRes1)) : 0;  // residual bits per dimension
  // TMEM columns of one decoded tile (fp16 pairs): d, or 2d for [hi | lo] rows
  const int acols = a.d / 2 * (SPLIT ? 2 : 1);
  const int S = a.nslot;
  const int n_cb = RES ? 0 : a.M * a.K * a.dsub;  // codebook elements (one table; the lo table follows)
  const TrLayout L = tr_layout(N, a.d, RES ? tr_res_bytes(S, a.d, NB) : static_cast<uint32_t>(n_cb * 2 * (SPLIT ? 2 : 1)), S);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t b_s = sbase + L.b_off;
  const uint32_t bar_s = sbase + L.bar_off;
  auto afull_bar = [&](int s) { return bar_s + 8u * s; };
  auto accf_bar = [&](int s) { return bar_s + 8u * (S + s); };
  auto free_bar = [&](int s) { return bar_s + 8u * (2 * S + s); };
  const uint32_t done_bar = bar_s + 8u * (3 * S);
  TrMisc* misc = reinterpret_cast<TrMisc*>(smem + L.misc_off);
  volatile int* abort_flag = &misc->abort;
  __half* cbs = reinterpret_cast<__half*>(smem + L.cb_off);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const DocLayout docs = a.docs;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(afull_bar(s), 8);  // the two decoder warps of each lane quarter
      mbar_init(accf_bar(s), 1);
      mbar_init(free_bar(s), Shape::kEpiWarps);
    }
    // the MMA-issuing threads commit to done_bar once each at the end
    mbar_init(done_bar, Shape::kMmaInDecoder ? 8 : 1);
    for (int i = 0; i < 8; ++i) misc->arrivals[i] = 0u;
    misc->abort = (sbase & 1023u) ? 1 : 0;  // SWIZZLE_128B needs a 1024-aligned base
    misc->never = 0;
    if (misc->abort) atomicCAS(a.err, 0u, kDevErrTimeout | 31u);
    fence_mbar_init();
  }
  if (warp == 0) {
    // This CTA's document-aligned token range, and its four document-aligned quarters.
    const int range = blockIdx.x;
    const int64_t t_first = docs.start(0);
    const int64_t span = docs.start(docs.n_docs) - t_first;
    const int64_t doc_lo = (range == 0) ? 0 : warp_lower_bound(docs, t_first + span * range / a.n_ranges);
    int64_t doc_hi = (range == a.n_ranges - 1)
                         ? docs.n_docs
                         : warp_lower_bound(docs, t_first + span * (range + 1) / a.n_ranges);
    if (doc_hi < doc_lo) doc_hi = doc_lo;
    const int64_t tok_lo = docs.start(doc_lo), tok_hi = docs.start(doc_hi);
    int64_t sd[5];
    sd[0] = doc_lo;
    sd[4] = doc_hi;
    for (int q = 1; q < 4; ++q) {
      int64_t x = warp_lower_bound(docs, tok_lo + (tok_hi - tok_lo) * q / 4);
      x = x < sd[q - 1] ? sd[q - 1] : x;
      sd[q] = x > doc_hi ? doc_hi : x;
    }
    if (lane == 0) {
      for (int q = 0; q <= 4; ++q) misc->sub_doc[q] = sd[q];
      misc->n_tiles = 0;
    }
  }
  // Stage the codebook as fp16 (PQ) or the bucket-weight table (residual), and the query rows as
  // the swizzled B operand (every thread helps).
  {
    if constexpr (RES) {
      // entry e (4 residual bits, most significant first = the lowest bit position) holds the
      // weights of the G = 4 / NB dimensions those bits encode: dimension g's bucket index has
      // bit k = bit 3 - (g NB + k) of e
      constexpr int G = 4 / NB;
      float* tab = reinterpret_cast<float*>(smem + L.cb_off);
      for (int i = threadIdx.x; i < 16 * G; i += blockDim.x) {
        const int e = i / G, g = i - e * G;
        int b = 0;
        for (int k = 0; k < NB; ++k) b |= ((e >> (3 - (g * NB + k))) & 1) << k;
        tab[i] = __ldg(a.bucket_w + b);
      }
    }
    const int n = n_cb;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      float v;
      if (a.cb_dtype == TMS_F16) v = __half2float(reinterpret_cast<const __half*>(a.codebook)[i]);
      else if (a.cb_dtype == TMS_BF16) v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.codebook)[i]);
      else v = reinterpret_cast<const float*>(a.codebook)[i];
      const __half hi = __float2half_rn(v);
      cbs[i] = hi;
      // the rounding error of hi, itself rounded to fp16: hi + lo carries ~22 significant bits
      if constexpr (SPLIT) cbs[n + i] = __float2half_rn(v - __half2float(hi));
    }
    const int upr = a.d / 8;  // 16-byte units per query row
    for (int i = threadIdx.x; i < N * upr; i += blockDim.x) {
      const int n_row = i / upr, u = i - n_row * upr;
      const int c = n_row >> 5;
      const int qi = c / a.nchunk;
      const int rq = (c - qi * a.nchunk) * 32 + (n_row & 31);
      uint4 val = make_uint4(0, 0, 0, 0);
      if (rq < a.nq && c < a.n_chunks)  // three chunks run on the four-chunk kernel: zero rows
        val = __ldg(reinterpret_cast<const uint4*>(a.Q + (static_cast<int64_t>(qi) * a.nq + rq) * a.d) + u);
      const uint32_t off = static_cast<uint32_t>((u >> 3) * N * 128 + n_row * 128) +
                           ((static_cast<uint32_t>(u & 7) ^ static_cast<uint32_t>(n_row & 7)) << 4);
      *reinterpret_cast<uint4*>(smem + L.b_off + off) = val;
    }
    fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core's reads
  }
  __syncthreads();
  if (warp < 4) {
    // tiles = the longest lane stream: the sum of the lengths of lane l's documents
    const int64_t first = misc->sub_doc[warp];
    const int ndq = static_cast<int>(misc->sub_doc[warp + 1] - first);
    LaneDocs<false> ld;
    ld.first = first;
    ld.ndq = ndq;
    uint32_t t = 0;
#pragma unroll 4
    for (int dd = lane; dd < ndq; dd += 32) {
      int64_t st;
      t += static_cast<uint32_t>(ld.fetch(docs, dd, st));
      t = t > (1u << 30) ? (1u << 30) : t;  // malformed offsets: bounded, never read past `codes`
    }
    t = __reduce_max_sync(0xffffffffu, t);
    if (lane == 0) atomicMax(&misc->n_tiles, static_cast<int>(t));
  }
  if (warp == Shape::kTmemWarp) {
    tmem_alloc(smem_u32(&misc->tmem), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint32_t tmem_base = misc->tmem;
  const uint64_t tmo = a.timeout_ns;
  const int n_tiles = misc->n_tiles;
  // slot s: decoded tile at columns [s*acols, (s+1)*acols), accumulator after all the A columns
  auto a_col = [&](int s) { return static_cast<uint32_t>(s * acols); };
  auto acc_col = [&](int s) { return static_cast<uint32_t>(S * acols + s * N); };

  // One thread, once tile j's decoded rows are all in TMEM: S^T = tile . Q^T.
  auto mma_tile = [&](int s) {
    const uint32_t idesc = make_idesc(128, N, 0u);
    // split codebook: K runs over [hi | lo] columns of A against the query rows twice
    const int kd = a.d / 16;
    for (int k = 0; k < acols / 8; ++k) {
      const int kq = (SPLIT && k >= kd) ? k - kd : k;
      const uint64_t bd = sw128_kmajor_desc(b_s + static_cast<uint32_t>((kq >> 2) * N * 128 + (kq & 3) * 32));
      mma_f16_ts(tmem_base + acc_col(s), tmem_base + a_col(s) + 8u * k, bd, idesc, k != 0);
    }
    mma_commit(accf_bar(s));
  };
  auto issue_tile = [&](int j) -> bool {
    const int s = j % S;
    if (!mbar_wait(afull_bar(s), (j / S) & 1u, abort_flag, tmo, a.err, 21)) return false;
    tc_fence_after();
    mma_tile(s);
    return true;
  };
  // every MMA the issuing thread launched lands before TMEM is released (bounded by time only)
  auto drain_mma = [&]() {
    mma_commit(done_bar);
    mbar_wait(done_bar, 0, &misc->never, tmo, a.err, 22);
  };

  const bool roles_run = !*abort_flag;
  if (!roles_run) {
    // misaligned shared memory: no role runs (the error word says why)
  } else if (!Shape::kMmaInDecoder && warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      for (int j = 0; j < n_tiles; ++j)
        if (!issue_tile(j)) break;
      drain_mma();
    }
  } else if (warp >= kTrDecWarp0 && warp < kTrEpiWarp0) {
    // ------------------------------------------------------------------ decoders
    // Warp (q, hp) rebuilds, for every tile, the 64-element column blocks h = hp, hp + 2, ... of
    // the 32 token rows of lane quarter q (one tcgen05.st of 32 lanes x 32 columns per block);
    // lane l's row is the next token of its document stream.
    const int q = warp & 3;
    const int hp = (warp - kTrDecWarp0) >> 2;
    const uint32_t t_quarter = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    auto nothing = [](int) {};
    if constexpr (RES) {
    // Residual decoding: warp hp rebuilds dimensions [hp d/2, (hp + 1) d/2) of its 32 tokens from
    // the centroid row and the residual bits (weights from the 16-entry table, 4 bits at a time),
    // rounds them once to fp16 into TMEM, and leaves the half's sum of squares in shared memory:
    // the epilogue scales each token's products by its inverse norm. Each lane copies its token's
    // centroid half-row (read through L2) and residual half-row into the warp's ring with cp.async
    // kTrResRing tiles ahead (its centroid id loaded a tile before that), so the decode reads
    // shared memory only.
    const int DH = a.d / 2;       // 32 or 64 dimensions
    const int UN = DH / 8;        // 16-byte centroid units: 4 or 8
    const int RW = DH * NB / 32;  // 32-bit residual words: 1 .. 8
    const int CP = 2 * DH + 16, PB = tr_res_pb(RW);
    const float* tab = reinterpret_cast<const float*>(smem + L.cb_off);
    float* nrm = reinterpret_cast<float*>(smem + L.cb_off + 256);
    const uint32_t slot_bytes = tr_res_slot(a.d, NB);
    uint8_t* ring = smem + L.cb_off + 256 + S * 1024 + (warp - kTrDecWarp0) * kTrResRing * slot_bytes;
    const uint32_t ring_s = smem_u32(ring);
    const uintptr_t rb_addr = reinterpret_cast<uintptr_t>(a.rbits);
    const bool wide16 = RW >= 4 && (rb_addr & 15) == 0;
    const bool wide8 = RW == 2 && (rb_addr & 7) == 0;
    LaneDocs<true> ls;
    ls.init(docs, misc->sub_doc[q], static_cast<int>(misc->sub_doc[q + 1] - misc->sub_doc[q]), lane, nothing);
    struct Ahead {
      int64_t pos;
      int32_t code;
      bool in;
    };
    auto take = [&]() -> Ahead {
      Ahead t;
      t.in = ls.active() && ls.pos >= 0 && ls.pos < a.n_tokens;
      t.pos = ls.pos;
      t.code = t.in ? __ldg(a.rcodes + ls.pos) : 0;
      ls.step(docs, nothing, nothing);
      return t;
    };
    // copies of tile t's rows into ring slot t % kTrResRing (one commit group per tile)
    // A lane whose stream has ended copies nothing: its ring slot keeps stale rows, which decode
    // into its own TMEM row only, and the epilogue never reads that lane (copying any fixed row
    // instead sent every idle lane of every SM to one L2 line).
    auto issue = [&](const Ahead& t, int r) {
      if (t.in) {
        int64_t c = t.code;
        c = c < 0 ? 0 : (c >= a.ncent ? a.ncent - 1 : c);  // never outside the table
        const __half* csrc = a.cent + c * a.d + hp * DH;
        const uint32_t cdst = ring_s + r * slot_bytes + lane * CP;
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (u < UN) cp_async16(cdst + 16u * u, csrc + 8 * u);
        const uint8_t* bsrc = a.rbits + t.pos * a.rbytes + hp * (a.rbytes / 2);
        const uint32_t bdst = ring_s + r * slot_bytes + 32 * CP + lane * PB;
        if (wide16) {
          for (int w4 = 0; w4 < RW / 4; ++w4) cp_async16(bdst + 16u * w4, bsrc + 16 * w4);
        } else if (wide8) {
          cp_async8(bdst, bsrc);
        } else {
          for (int w1 = 0; w1 < RW; ++w1) cp_async4(bdst + 4u * w1, bsrc + 4 * w1);
        }
      }
      cp_async_commit();
    };
    bool ok = !(a.debug_flags & 1);
    if (ok) {
#pragma unroll
      for (int t = 0; t < kTrResRing; ++t) {
        const Ahead A = take();
        if (t < n_tiles) issue(A, t);
        else cp_async_commit();
      }
    }
    Ahead C = take();  // the tile kTrResRing ahead of the decode
    for (int j = 0; ok && j < n_tiles; ++j) {
      const int s = j % S;
      const int r = j % kTrResRing;
      int w = 0;
      if (lane == 0) w = mbar_wait(free_bar(s), ((j / S) & 1u) ^ 1u, abort_flag, tmo, a.err, 23);
      if (!(ok = __shfl_sync(0xffffffffu, w, 0) != 0)) break;
      cp_async_wait_group<kTrResRing - 1>();  // this lane's copies of tile j have landed
      const uint8_t* crow = ring + r * slot_bytes + lane * CP;
      const uint8_t* brow = ring + r * slot_bytes + 32 * CP + lane * PB;
      uint32_t bits[8];
      if (RW >= 4) {
#pragma unroll
        for (int w4 = 0; w4 < 2; ++w4)
          if (4 * w4 < RW) {
            const uint4 v = *reinterpret_cast<const uint4*>(brow + 16 * w4);
            bits[4 * w4] = v.x;
            bits[4 * w4 + 1] = v.y;
            bits[4 * w4 + 2] = v.z;
            bits[4 * w4 + 3] = v.w;
          }
      } else if (RW == 2) {
        const uint2 v = *reinterpret_cast<const uint2*>(brow);
        bits[0] = v.x;
        bits[1] = v.y;
      } else {
        bits[0] = *reinterpret_cast<const uint32_t*>(brow);
      }
      uint32_t out[32];
      uint64_t ss = 0ull;  // a pair of partial sums of squares
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (u < UN) {
          // unit u: dimensions 8u .. 8u + 7 of the half = residual nibbles 2u NB .. 2u NB + 2NB - 1
          // (bit positions in order: the high nibble of a byte first)
          float wt[8];
#pragma unroll
          for (int k = 0; k < 2 * NB; ++k) {
            const int n = 2 * u * NB + k;
            const int byte = n >> 1;
            const uint32_t e = (bits[byte >> 2] >> (8 * (byte & 3) + ((n & 1) ? 0 : 4))) & 0xFu;
            if constexpr (NB == 1) {
              const float4 t4 = *reinterpret_cast<const float4*>(tab + 4 * e);
              wt[4 * k] = t4.x;
              wt[4 * k + 1] = t4.y;
              wt[4 * k + 2] = t4.z;
              wt[4 * k + 3] = t4.w;
            } else if constexpr (NB == 2) {
              const float2 t2 = *reinterpret_cast<const float2*>(tab + 2 * e);
              wt[2 * k] = t2.x;
              wt[2 * k + 1] = t2.y;
            } else {
              wt[k] = tab[e];
            }
          }
          const uint4 cu = *reinterpret_cast<const uint4*>(crow + 16 * u);
          const uint32_t cw[4] = {cu.x, cu.y, cu.z, cu.w};
#pragma unroll
          for (int p2 = 0; p2 < 4; ++p2) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&cw[p2]));
            const uint64_t x = f2_add(f2_pack(f.x, f.y), f2_pack(wt[2 * p2], wt[2 * p2 + 1]));
            ss = f2_fma(x, x, ss);
            const float2 v = f2_unpack(x);
            const __half2 h = __floats2half2_rn(v.x, v.y);
            out[4 * u + p2] = *reinterpret_cast<const uint32_t*>(&h);
          }
        }
      }
      if (DH == 64) tmem_st32(t_quarter + a_col(s) + 32u * hp, out);
      else tmem_st16(t_quarter + a_col(s) + 16u * hp, out);
      const float2 sp = f2_unpack(ss);
      nrm[((s * 4 + q) * 2 + hp) * 32 + lane] = sp.x + sp.y;
      // slot r is read (the stores above consumed it): refill it with tile j + kTrResRing
      if (j + kTrResRing < n_tiles) issue(C, r);
      else cp_async_commit();
      C = take();
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (!Shape::kMmaInDecoder) {
        if (lane == 0) mbar_arrive(afull_bar(s));
      } else if (lane == 0 && (count_arrival(&misc->arrivals[s]) & 7u) == 7u) {
        tc_fence_after();
        mma_tile(s);
      }
    }
    cp_async_wait_all();  // no copy into the ring outlives the kernel
    } else {
    // d = 128, M = 16, dsub = 8: warp hp needs code bytes [8 hp, 8 hp + 8) of each token
    const bool fast = (a.M == 16) && (a.dsub == 8) && ((reinterpret_cast<uintptr_t>(a.codes) & 15) == 0);
    const uint32_t kmax = static_cast<uint32_t>(a.K - 1);
    // The stream runs two tiles ahead of the decode in the fast case (codes of the next two
    // tiles in flight), level with it otherwise (codes read inside the decode).
    LaneDocs<true> ls;
    ls.init(docs, misc->sub_doc[q], static_cast<int>(misc->sub_doc[q + 1] - misc->sub_doc[q]), lane, nothing);
    auto load_codes = [&]() -> uint2 {
      const bool in = ls.active() && ls.pos >= 0 && ls.pos < a.n_tokens;
      const uint2 c = in ? __ldg(reinterpret_cast<const uint2*>(a.codes + ls.pos * 16 + 8 * hp)) : make_uint2(0, 0);
      ls.step(docs, nothing, nothing);
      return c;
    };
    uint2 c_n1 = make_uint2(0, 0), c_n2 = make_uint2(0, 0);
    if (fast) {
      c_n1 = load_codes();
      c_n2 = load_codes();
    }
    bool ok = !(a.debug_flags & 1);
    for (int j = 0; ok && j < n_tiles; ++j) {
      const uint2 cc = c_n1;
      c_n1 = c_n2;
      if (fast) c_n2 = load_codes();
      const int s = j % S;
      int w = 0;
      if (lane == 0) w = mbar_wait(free_bar(s), ((j / S) & 1u) ^ 1u, abort_flag, tmo, a.err, 23);
      if (!(ok = __shfl_sync(0xffffffffu, w, 0) != 0)) break;
      const int hblocks = a.d / 64;
      if (fast) {
        // d = 128: this warp's block h = hp holds subspaces 8 hp .. 8 hp + 7. Lanes whose stream
        // has ended decode code 0 (load_codes) and the epilogue never reads them.
        // Split codebook: the lo row sits at a fixed offset from the hi row, so one code and one
        // address serve both loads, and the lo values go to block hp + hblocks.
        const char* tab = reinterpret_cast<const char*>(cbs);
        uint32_t off[8];  // byte offsets of the 8 codebook rows in the hi table
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          uint32_t code = ((i < 4 ? cc.x : cc.y) >> (8 * (i & 3))) & 0xffu;
          code = min(code, kmax);  // never read past the codebook
          off[i] = (static_cast<uint32_t>((8 * hp + i) * a.K) + code) * 16u;
        }
#pragma unroll
        for (int half = 0; half < (SPLIT ? 2 : 1); ++half) {
          const char* t = tab + (half ? n_cb * 2 : 0);
          uint32_t r[32];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint4 e = *reinterpret_cast<const uint4*>(t + off[i]);
            r[4 * i] = e.x;
            r[4 * i + 1] = e.y;
            r[4 * i + 2] = e.z;
            r[4 * i + 3] = e.w;
          }
          tmem_st32(t_quarter + a_col(s) + 32u * (hp + half * hblocks), r);
        }
      } else {
        const int64_t tok = ls.pos;
        const bool valid = ls.active() && tok >= 0 && tok < a.n_tokens;
        for (int h = hp; h < hblocks * (SPLIT ? 2 : 1); h += 2) {
          // block h of the decoded row: column block hh of the hi table, or of the lo table
          const bool lo_half = SPLIT && h >= hblocks;
          const int hh = lo_half ? h - hblocks : h;
          const __half* tab = lo_half ? cbs + n_cb : cbs;
          uint32_t r[32];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int col = 8 * (8 * hh + i);  // first element of this 16-byte unit
            const int m = col / a.dsub, part = col - m * a.dsub;
            uint4 e = make_uint4(0, 0, 0, 0);
            if (valid) {
              const uint32_t code = min(static_cast<uint32_t>(__ldg(a.codes + tok * a.M + m)), kmax);
              e = *reinterpret_cast<const uint4*>(tab + (m * a.K + code) * a.dsub + part);
            }
            r[4 * i] = e.x;
            r[4 * i + 1] = e.y;
            r[4 * i + 2] = e.z;
            r[4 * i + 3] = e.w;
          }
          tmem_st32(t_quarter + a_col(s) + 32u * h, r);
        }
        ls.step(docs, nothing, nothing);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (!Shape::kMmaInDecoder) {
        if (lane == 0) mbar_arrive(afull_bar(s));
      } else if (lane == 0 && (count_arrival(&misc->arrivals[s]) & 7u) == 7u) {
        tc_fence_after();
        mma_tile(s);
      }
    }
    }
    // each decoder warp commits once: done_bar completes when every MMA it issued has landed
    if (Shape::kMmaInDecoder && lane == 0) mma_commit(done_bar);
  } else if (warp >= kTrEpiWarp0 || (Shape::kEpiWarps == 8 && warp < 4)) {
    // ------------------------------------------------------------------ epilogue
    // Lane l keeps, per query row i, the running max acc[c][i] over the tokens of its current
    // document (one per tile); when the document's last token has been merged it sums the rows
    // (in order i = 0, 1, ...) and stores the score. Empty documents score -inf.
    const int q = warp & 3;
    const uint32_t t_quarter = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    // this warp's chunks: cbase .. cbase + EC - 1
    constexpr int EC = Shape::kEpiChunks;
    const int cbase = (NCH > 2 && warp < 4) ? EC : 0;
    // Padded query rows are zero, so their row maximum over a non-empty document is exactly 0 and
    // the score sums all 32 rows of a chunk; every stored chunk has a real row, so an empty
    // document scores -inf.
    float acc[EC][32];
#pragma unroll
    for (int c = 0; c < EC; ++c)
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[c][i] = kTrNegInf;
    auto store = [&](int c, int dd, float x) {
      if (cbase + c < a.n_chunks)
        a.out[static_cast<int64_t>(cbase + c) * docs.n_docs + misc->sub_doc[q] + dd] = x;
    };
    auto on_empty = [&](int dd) {
#pragma unroll
      for (int c = 0; c < EC; ++c) store(c, dd, kTrNegInf);
    };
    auto nothing = [](int) {};
    LaneDocs<false> ls;
    ls.init(docs, misc->sub_doc[q], static_cast<int>(misc->sub_doc[q + 1] - misc->sub_doc[q]), lane, on_empty);
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int s = j % S;
      int w = 0;
      if (lane == 0) w = mbar_wait(accf_bar(s), (j / S) & 1u, abort_flag, tmo, a.err, 24);
      if (!(ok = __shfl_sync(0xffffffffu, w, 0) != 0)) break;
      tc_fence_after();
      const bool act = ls.active();
      // residual corpora scaled to unit length: this lane's token's inverse norm, from the two
      // decoder halves' sums of squares (read before the slot is handed back; the decoders
      // published them before their tile hand-off, which this acquires)
      float inv = 1.0f;
      if (RES && a.normalize) {
        if (Shape::kMmaInDecoder) {
          cuda::atomic_ref<uint32_t, cuda::thread_scope_block> ctr(misc->arrivals[s]);
          (void)ctr.load(cuda::memory_order_acquire);
        } else {
          if (lane == 0) w = mbar_wait(afull_bar(s), (j / S) & 1u, abort_flag, tmo, a.err, 25);
          if (!(ok = __shfl_sync(0xffffffffu, w, 0) != 0)) break;
          __syncwarp();  // lane 0's acquire orders the other lanes' reads below
        }
        const float* nrm = reinterpret_cast<const float*>(smem + L.cb_off + 256) + (s * 4 + q) * 64 + lane;
        const float ssq = nrm[0] + nrm[32];
        inv = ssq > 0.0f ? rsqrtf(ssq) : 0.0f;
      }
#pragma unroll
      for (int c = 0; c < EC; ++c) {
        uint32_t r[32];
        tmem_ld32_async(t_quarter + acc_col(s) + 32u * (cbase + c), r);
        tmem_wait_ld32(r);
        if (c == EC - 1) {  // the slot's last read: hand it back before the math
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(free_bar(s));
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float v = RES ? __uint_as_float(r[i]) * inv : __uint_as_float(r[i]);
          acc[c][i] = act ? fmaxf(acc[c][i], v) : acc[c][i];
        }
      }
      // a document ends on this lane: its scores (summed by the whole warp, a uniform branch, so
      // that no divergent region holds the accumulators), then the stream moves on
      const bool ends = act && ls.rem == 1;
      if (__any_sync(0xffffffffu, ends)) {
#pragma unroll
        for (int c = 0; c < EC; ++c) {
          float x = 0.0f;
#pragma unroll
          for (int i = 0; i < 32; ++i) x += acc[c][i];
          if (ends) store(c, ls.d, x);
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[c][i] = ends ? kTrNegInf : acc[c][i];
        }
      }
      ls.step(docs, nothing, on_empty);
      __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == Shape::kTmemWarp) {
    // decoder-issued MMAs: all eight commits are in (before the barrier); wait for the MMAs
    if (Shape::kMmaInDecoder && roles_run && lane == 0) mbar_wait(done_bar, 0, &misc->never, tmo, a.err, 22);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

__global__ void tr_sum_chunks_kernel(const float* __restrict__ partial, float* __restrict__ out,
                                     int64_t n_queries, int64_t n_docs, int nchunk) {
  const int64_t total = n_queries * n_docs;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t qq = i / n_docs;
    const int64_t dd = i - qq * n_docs;
    float s = 0.0f;
    for (int p = 0; p < nchunk; ++p) s += partial[(qq * nchunk + p) * n_docs + dd];
    out[i] = s;
  }
}

}  // namespace

size_t pq_tokrows_workspace_size(int64_t n_queries, int64_t nq, int64_t n_docs) {
  const int64_t nchunk = (nq + 31) / 32;
  return nchunk > 1 ? align_up(static_cast<size_t>(n_queries * nchunk * n_docs) * 4, 256) : 0;
}

namespace {

using TrKernel = void (*)(TrArgs);
template <int MODE>
TrKernel tr_kernel(int nch) {
  return nch == 1 ? pq_tokrows_kernel<1, MODE> : (nch == 2 ? pq_tokrows_kernel<2, MODE> : pq_tokrows_kernel<4, MODE>);
}

// the epilogue walks 32-bit positions (token and document indices)
constexpr int64_t kTrMax32 = 0x7fffffffLL - 64;

// Shared by the PQ and residual entry points: a.d, a.nq and the source fields set by the caller.
int tr_launch(TrArgs& a, int mode, int64_t n_queries, int64_t nq, int64_t n_tokens,
              const int64_t* doc_offsets, int64_t n_docs, int64_t nd_uniform, float* out,
              void* workspace, size_t workspace_bytes, cudaStream_t st, int acols,
              uint32_t fixed_bytes) {
  const int64_t nchunk = (nq + 31) / 32;
  const int64_t chunks = n_queries * nchunk;
  if (chunks < 1 || chunks > kTrMaxChunks || n_tokens > kTrMax32 || n_docs > kTrMax32 || n_tokens <= 0)
    return TMS_ERR_UNSUPPORTED;
  int status = TMS_OK;
  const DeviceInfo* dev = current_device_info(&status);
  if (!dev) return status;
  // the kernel's query tile is NCH x 32 rows: three chunks run on the four-chunk kernel
  const int nch = chunks > 2 ? 4 : static_cast<int>(chunks);
  const int N = nch * 32;
  // as many slots as TMEM holds: a hand-off through an mbarrier takes ~500 cycles, so several
  // tiles must be in flight between the decoders, the MMA and the epilogue
  int nslot = 512 / (acols + N);
  if (nslot > 8) nslot = 8;
  if (nslot < 2 || nslot * (acols + N) > 512) return TMS_ERR_UNSUPPORTED;
  const size_t need = pq_tokrows_workspace_size(n_queries, nq, n_docs);
  if (need && (!workspace || workspace_bytes < need)) return TMS_ERR_WORKSPACE;
  a.docs.offsets = doc_offsets;
  a.docs.n_docs = n_docs;
  a.docs.nd = doc_offsets ? 0 : nd_uniform;
  a.n_tokens = n_tokens;
  a.out = nchunk > 1 ? static_cast<float*>(workspace) : out;
  a.err = dev->err_word;
  a.timeout_ns = wait_timeout_ns();
  a.nchunk = static_cast<int>(nchunk);
  a.n_chunks = static_cast<int>(chunks);
  a.nslot = nslot;
  a.debug_flags = debug_flags();
  // one CTA per SM (a persistent range each), fewer for small corpora
  int64_t ranges = dev->num_sms;
  const int64_t min_tiles = (n_tokens + 127) / 128;
  if (ranges > min_tiles) ranges = min_tiles;
  if (ranges > n_docs) ranges = n_docs;
  if (ranges < 1) ranges = 1;
  a.n_ranges = static_cast<int>(ranges);
  const uint32_t cb_bytes =
      mode >= kTrRes1 ? tr_res_bytes(nslot, a.d, 1 << (mode - kTrRes1)) : fixed_bytes;
  const TrLayout L = tr_layout(N, a.d, cb_bytes, nslot);
  // at least half the SM's shared memory: one CTA per SM, so the 512-column TMEM allocation
  // never waits for another CTA
  size_t smem = L.total;
  const size_t half = static_cast<size_t>(dev->max_smem_optin) / 2 + 1024;
  if (smem < half) smem = half;
  if (static_cast<int>(smem) > dev->max_smem_optin) return TMS_ERR_UNSUPPORTED;
  TrKernel kern = nullptr;
  switch (mode) {
    case kTrPq: kern = tr_kernel<kTrPq>(nch); break;
    case kTrPqSplit: kern = tr_kernel<kTrPqSplit>(nch); break;
    case kTrRes1: kern = tr_kernel<kTrRes1>(nch); break;
    case kTrRes2: kern = tr_kernel<kTrRes2>(nch); break;
    default: kern = tr_kernel<kTrRes4>(nch); break;
  }
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return TMS_ERR_CUDA;
  kern<<<static_cast<unsigned>(ranges), kTrThreads, smem, st>>>(a);
  if (cudaGetLastError() != cudaSuccess) return TMS_ERR_CUDA;
  if (nchunk == 1) return TMS_OK;
  const int64_t total = n_queries * n_docs;
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > dev->num_sms * 8) blocks = dev->num_sms * 8;
  tr_sum_chunks_kernel<<<blocks, 256, 0, st>>>(static_cast<const float*>(workspace), out, n_queries,
                                               n_docs, static_cast<int>(nchunk));
  return cuda_status(cudaGetLastError());
}

}  // namespace

int pq_tokrows_maxsim(const void* Q, int64_t n_queries, int64_t nq, const void* codebook,
                      int cb_dtype, int64_t M, int64_t K, int64_t dsub, const uint8_t* codes,
                      int64_t n_tokens, const int64_t* doc_offsets, int64_t n_docs,
                      int64_t nd_uniform, float* out, void* workspace, size_t workspace_bytes,
                      cudaStream_t st, bool split) {
  const int64_t d = M * dsub;
  const size_t cb_bytes = static_cast<size_t>(M * K * dsub) * 2 * (split ? 2 : 1);
  if (d % 64 != 0 || d > 256 || dsub % 8 != 0 || K < 1 || K > 256 ||
      cb_bytes > (split ? 128 : 96) * 1024 || (reinterpret_cast<uintptr_t>(Q) & 15))
    return TMS_ERR_UNSUPPORTED;
  TrArgs a = {};
  a.codes = codes;
  a.Q = static_cast<const __half*>(Q);
  a.codebook = codebook;
  a.cb_dtype = cb_dtype;
  a.M = static_cast<int>(M);
  a.K = static_cast<int>(K);
  a.dsub = static_cast<int>(dsub);
  a.d = static_cast<int>(d);
  a.nq = static_cast<int>(nq);
  return tr_launch(a, split ? kTrPqSplit : kTrPq, n_queries, nq, n_tokens, doc_offsets, n_docs,
                   nd_uniform, out, workspace, workspace_bytes, st,
                   static_cast<int>(d / 2) * (split ? 2 : 1), static_cast<uint32_t>(cb_bytes));
}

int res_tokrows_maxsim(const void* Q, int64_t n_queries, int64_t nq, int64_t d,
                       const void* centroids, int64_t n_centroids, const int32_t* codes,
                       const uint8_t* residuals, const float* bucket_weights, int nbits,
                       int normalize, int64_t n_tokens, const int64_t* doc_offsets, int64_t n_docs,
                       int64_t nd_uniform, float* out, void* workspace, size_t workspace_bytes,
                       cudaStream_t st) {
  if ((d != 64 && d != 128) || (nbits != 1 && nbits != 2 && nbits != 4) || n_centroids < 1 ||
      (reinterpret_cast<uintptr_t>(Q) & 15) || (reinterpret_cast<uintptr_t>(centroids) & 15) ||
      (reinterpret_cast<uintptr_t>(residuals) & 3) || (reinterpret_cast<uintptr_t>(codes) & 3))
    return TMS_ERR_UNSUPPORTED;
  TrArgs a = {};
  a.Q = static_cast<const __half*>(Q);
  a.d = static_cast<int>(d);
  a.nq = static_cast<int>(nq);
  a.cent = static_cast<const __half*>(centroids);
  a.ncent = n_centroids;
  a.rcodes = codes;
  a.rbits = residuals;
  a.bucket_w = bucket_weights;
  a.rbytes = static_cast<int>(d * nbits / 8);
  a.normalize = normalize ? 1 : 0;
  const int mode = nbits == 1 ? kTrRes1 : (nbits == 2 ? kTrRes2 : kTrRes4);
  return tr_launch(a, mode, n_queries, nq, n_tokens, doc_offsets, n_docs, nd_uniform, out,
                   workspace, workspace_bytes, st, static_cast<int>(d / 2), 0u);
}

}  // namespace tms
