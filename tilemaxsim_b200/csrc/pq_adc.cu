// pq_adc.cu -- MaxSim straight from product-quantization codes (asymmetric distance computation).
//
//   table[q, i, m, k] = <Q[q, i, m*dsub:(m+1)*dsub], C[m, k, :]>           (fp32)
//   score[q, doc]    = sum_i max_{j in doc} sum_m table[q, i, m, codes[j, m]]
//
// Reference: src/flash_pqsim_kernel.py:31-67 (_build_distance_table_kernel), :127-173
// (_flash_pqsim_batched_score_kernel: per (query token, doc) running max of the m-ordered table
// sums) and :213-280 (score_batch sums the per-token maxima; score_single for one document).
//
// B200 design: one CTA owns a slice of QS query tokens of one query and a range of documents. It
// builds that slice's table in shared memory as T[m][k][QS] (fp32, so one code byte fetches the
// entries of all QS query tokens with 128-bit shared loads), then a warp scores one document at a
// time: lanes stride over the document's tokens, read each token's M code bytes with 16-byte
// vector loads, accumulate the M table entries per query token in m order (the reference's
// summation order), keep per-lane running maxima, and reduce them across the warp when the
// document ends. Codes are never decoded to vectors and the table never touches HBM.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "tms_device.cuh"
#include "tms_internal.h"

namespace tms {
namespace {

constexpr int kPqThreads = 512;
constexpr int kPqTableBudget = 200 * 1024;
constexpr float kNegInfPq = -__builtin_huge_valf();

// Three-input fp32 max (PTX max.f32 with three sources, sm_100a).
__device__ __forceinline__ float fmax3(float x, float y, float z) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(x), "f"(y), "f"(z));
  return r;
}

__device__ __forceinline__ float load_elem(const void* p, int dtype, int64_t i) {
  if (dtype == TMS_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  if (dtype == TMS_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

// table[((q*nq + i) * M + m) * K + k] in fp32, one thread per entry (the reference's layout).
__global__ void pq_table_kernel(const void* __restrict__ Q, int q_dtype, int64_t n_rows,
                                const void* __restrict__ cb, int cb_dtype, int M, int K, int dsub,
                                float* __restrict__ table) {
  const int64_t total = n_rows * M * K;
  const int d = M * dsub;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = e / (static_cast<int64_t>(M) * K);
    const int rem = static_cast<int>(e - r * M * K);
    const int m = rem / K, k = rem - m * K;
    float acc = 0.0f;
    for (int t = 0; t < dsub; ++t)
      acc = fmaf(load_elem(Q, q_dtype, r * d + m * dsub + t),
                 load_elem(cb, cb_dtype, (static_cast<int64_t>(m) * K + k) * dsub + t), acc);
    table[e] = acc;
  }
}

struct PqArgs {
  const void* Q;
  const void* cb;
  const uint8_t* codes;
  int64_t n_tokens;  // rows of codes: token ranges are clamped to [0, n_tokens)
  DocLayout docs;
  float* out;  // (n_queries * nslice, n_docs): slice partial scores (final scores if nslice == 1)
  int q_dtype, cb_dtype;
  int nq, M, K, dsub;
  int nslice;      // query-token slices per query
  int n_doc_parts;
};

template <int QS, bool M16>
__global__ void __launch_bounds__(kPqThreads)
    pq_maxsim_kernel(const PqArgs a) {
  extern __shared__ __align__(16) float tbl[];  // [M][K][QS]
  const int slice_id = blockIdx.x / a.n_doc_parts;
  const int part = blockIdx.x - slice_id * a.n_doc_parts;
  const int q = slice_id / a.nslice;
  const int i0 = (slice_id - q * a.nslice) * QS;
  const int d = a.M * a.dsub;

  // Build T[m][k][s] = <Q[q, i0+s, m-slice], C[m, k]> (zero for query tokens past nq).
  const int n_ent = a.M * a.K * QS;
  for (int e = threadIdx.x; e < n_ent; e += blockDim.x) {
    const int s = e % QS;
    const int mk = e / QS;
    const int m = mk / a.K, k = mk - m * a.K;
    const int i = i0 + s;
    float acc = 0.0f;
    if (i < a.nq) {
      const int64_t qrow = (static_cast<int64_t>(q) * a.nq + i) * d + m * a.dsub;
      const int64_t crow = (static_cast<int64_t>(m) * a.K + k) * a.dsub;
      for (int t = 0; t < a.dsub; ++t)
        acc = fmaf(load_elem(a.Q, a.q_dtype, qrow + t), load_elem(a.cb, a.cb_dtype, crow + t), acc);
    }
    tbl[e] = acc;
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_warps = blockDim.x >> 5;
  const int64_t n_docs = a.docs.n_docs;
  const int64_t doc_begin = n_docs * part / a.n_doc_parts;
  const int64_t doc_end = n_docs * (part + 1) / a.n_doc_parts;
  const int ns = min(QS, a.nq - i0);
  const uint32_t kmax = static_cast<uint32_t>(a.K - 1);
  for (int64_t doc = doc_begin + warp; doc < doc_end; doc += n_warps) {
    // clamped to the code rows that exist, so malformed offsets never read outside `codes`
    const int64_t t_lo = max(min(a.docs.start(doc), a.n_tokens), int64_t(0));
    const int64_t t_hi = max(min(a.docs.start(doc + 1), a.n_tokens), t_lo);
    float run[QS];
#pragma unroll
    for (int s = 0; s < QS; ++s) run[s] = kNegInfPq;
    for (int64_t j = t_lo + lane; j < t_hi; j += 32) {
      float acc[QS];
#pragma unroll
      for (int s = 0; s < QS; ++s) acc[s] = 0.0f;
      const uint8_t* row = a.codes + j * a.M;
      if (M16) {
        const uint4 c4 = __ldg(reinterpret_cast<const uint4*>(row));
        const uint32_t w[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
        for (int m = 0; m < 16; ++m) {
          uint32_t code = (w[m >> 2] >> (8 * (m & 3))) & 0xffu;
          if (kmax < 255u) code = min(code, kmax);  // a code >= K never reads past the table
          const float* e = tbl + (m * a.K + code) * QS;
          if (QS % 4 == 0) {
#pragma unroll
            for (int s = 0; s < QS; s += 4) {
              const float4 t = *reinterpret_cast<const float4*>(e + s);
              acc[s] += t.x;
              acc[s + 1] += t.y;
              acc[s + 2] += t.z;
              acc[s + 3] += t.w;
            }
          } else {
#pragma unroll
            for (int s = 0; s < QS; ++s) acc[s] += e[s];
          }
        }
      } else {
        for (int m = 0; m < a.M; ++m) {
          const uint32_t code = min(static_cast<uint32_t>(__ldg(row + m)), kmax);
          const float* e = tbl + (m * a.K + code) * QS;
#pragma unroll
          for (int s = 0; s < QS; ++s) acc[s] += e[s];
        }
      }
#pragma unroll
      for (int s = 0; s < QS; ++s) run[s] = fmaxf(run[s], acc[s]);
    }
    float total = 0.0f;
#pragma unroll
    for (int s = 0; s < QS; ++s) {
      const float mx = warp_max(run[s]);
      if (s < ns) total += mx;
    }
    if (lane == 0) a.out[static_cast<int64_t>(slice_id) * n_docs + doc] = total;
  }
}

// Bank-conflict-free table lookups (M = 8 or 16).
//
// The kernel above gives each lane its own document token, so the 32 lanes of a load read table
// rows chosen by 32 random codes and collide in the shared-memory banks (about 2.4 wavefronts per
// ideal one at M = 16). Here the lanes of a warp work on the SAME four tokens: lane = (g, i) with
// i = lane & 7 the query token of the slice and g = lane >> 3 one of four subspace groups
// (subspaces m = A g + aa, aa = 0 .. A-1, A = M / 4: the group's A consecutive code bytes). The
// table is stored as rows of 32 floats,
//
//     T4[aa][k][8 g + i] = <Q[q, i0 + i, m-slice], C[m, k]>,   m = A g + aa,
//
// (rows of code bytes aa = 2 rp and 2 rp + 1 interleaved in 256-byte row pairs, so that one byte
// permute turns a code byte into the entry's offset),
// so at every step aa the four lane groups read four rows picked by four different codes, but
// each group only ever touches its own eight banks (8 g .. 8 g + 7): every load is one wavefront,
// whatever the codes are. A lane group loads only its own A code bytes of a token (one 4- or
// 2-byte load; the warp's four groups read four tokens inside one 64-byte span), sums its A
// subspaces, and a two-round reduce-scatter over the lane groups (3 shuffles per four tokens)
// leaves the full sum of token j0 + g in lane group g, which keeps a running max over its tokens
// of the document. At the document's end the groups' maxima are merged (2 shuffles) and the 8
// query tokens summed (3 shuffles). The m-summation order is (groups of A subspaces, then across
// groups) instead of the reference's m = 0, 1, 2, ...: the sums differ only by fp32 rounding.
constexpr int kLut4Threads = 512;

template <int A, int KT>  // A = M / 4 table rows per token; KT = K when it is 256, else 0
__global__ void __launch_bounds__(kLut4Threads, 1) pq_lut4_kernel(const PqArgs a) {
  extern __shared__ __align__(128) float tbl4[];  // [A / 2][K][2][32]
  const int n_slices = gridDim.x / a.n_doc_parts;
  // consecutive CTAs share a document range (and its codes in L2) and differ in query slice
  const int slice_id = blockIdx.x % n_slices;
  const int part = blockIdx.x / n_slices;
  const int q = slice_id / a.nslice;
  const int i0 = (slice_id - q * a.nslice) * 8;
  const int d = a.M * a.dsub;
  const int K = KT ? KT : a.K;

  // entry e = ((rp * K + k) * 2 + half) * 32 + col holds subspace byte aa = 2 rp + half
  for (int e = threadIdx.x; e < A * K * 32; e += blockDim.x) {
    const int col = e & 31;
    const int half = (e >> 5) & 1;
    const int rk = e >> 6;
    const int rp = rk / K, k = rk - rp * K;
    const int aa = 2 * rp + half;
    const int m = A * (col >> 3) + aa;
    const int i = i0 + (col & 7);
    float acc = 0.0f;
    if (i < a.nq) {
      const int64_t qrow = (static_cast<int64_t>(q) * a.nq + i) * d + m * a.dsub;
      const int64_t crow = (static_cast<int64_t>(m) * K + k) * a.dsub;
      for (int t = 0; t < a.dsub; ++t)
        acc = fmaf(load_elem(a.Q, a.q_dtype, qrow + t), load_elem(a.cb, a.cb_dtype, crow + t), acc);
    }
    tbl4[e] = acc;
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 3, i = lane & 7;
  const int n_warps = blockDim.x >> 5;
  const int64_t n_docs = a.docs.n_docs;
  const int64_t doc_begin = n_docs * part / a.n_doc_parts;
  const int64_t doc_end = n_docs * (part + 1) / a.n_doc_parts;
  const int ns = min(8, a.nq - i0);
  const uint32_t kmax = static_cast<uint32_t>(K - 1);
  // Byte offset of this lane's entry for code byte aa inside its 256-byte row pair: code * 256
  // + lane * 4, built by one byte permute (byte 1 = the code, byte 0 = lane * 4 < 128, bytes 2-3
  // = zero bytes of lane4); the row pair and half go into the load's immediate offset.
  const uint32_t lane4 = static_cast<uint32_t>(lane) * 4u;
  auto row_off = [&](uint32_t w, int aa) -> uint32_t {
    if constexpr (KT == 256) {
      return __byte_perm(w, lane4, 0x5504u | (static_cast<uint32_t>(aa) << 4));
    } else {
      const uint32_t code = min((w >> (8 * aa)) & 0xffu, kmax);  // a code >= K never reads past the table
      return (code << 8) | lane4;
    }
  };
  const char* tb = reinterpret_cast<const char*>(tbl4);
  auto lookup = [&](int aa, uint32_t off) -> float {
    return *reinterpret_cast<const float*>(tb + static_cast<uint32_t>((aa >> 1) * K * 256 + (aa & 1) * 128) + off);
  };
  // Codes are staged per warp in shared memory, 32 tokens at a time: lane l loads token l's whole
  // code row with one coalesced load (the next 32 rows are in flight in registers meanwhile) and
  // stores it transposed, word g (code bytes A g .. A g + A - 1) into row g of the stage (rows 36
  // words apart, so the four rows start in different banks). Lane group g then reads its words of
  // four consecutive tokens with one vector load.
  using CodeWord = typename std::conditional<A == 4, uint32_t, uint16_t>::type;
  using CodeRow = typename std::conditional<A == 4, uint4, uint2>::type;
  using Word4 = typename std::conditional<A == 4, uint4, uint2>::type;  // 4 tokens' words
  constexpr int kStagePitch = 36 * 4 / A;  // CodeWords per stage row (144 bytes)
  CodeWord* const stage = reinterpret_cast<CodeWord*>(tbl4 + A * K * 32) + warp * 4 * kStagePitch;
  const Word4* const stage_g = reinterpret_cast<const Word4*>(stage + g * kStagePitch);
  auto word_of = [](const Word4& w, int u) -> uint32_t {  // token u's word of a 4-token vector
    if constexpr (A == 4) return u == 0 ? w.x : u == 1 ? w.y : u == 2 ? w.z : w.w;
    else return ((u < 2 ? w.x : w.y) >> (16 * (u & 1))) & 0xffffu;
  };
  auto row_word = [](const CodeRow& r, int gg) -> CodeWord {
    if constexpr (A == 4) return gg == 0 ? r.x : gg == 1 ? r.y : gg == 2 ? r.z : r.w;
    else return static_cast<CodeWord>(((gg < 2 ? r.x : r.y) >> (16 * (gg & 1))) & 0xffffu);
  };

  for (int64_t doc = doc_begin + warp; doc < doc_end; doc += n_warps) {
    // clamped to the code rows that exist, so malformed offsets never read outside `codes`
    const int64_t t_lo = max(min(a.docs.start(doc), a.n_tokens), int64_t(0));
    const int64_t t_hi = max(min(a.docs.start(doc + 1), a.n_tokens), t_lo);
    const int len = static_cast<int>(min(t_hi - t_lo, int64_t(0x7fffffff)));
    const CodeRow* rows = reinterpret_cast<const CodeRow*>(a.codes + t_lo * (4 * A));
    float run = kNegInfPq;
    const int last = len - 1;
    // the full sum of token j0 + g from this lane's partial sums p[t] of tokens j0 + (t ^ g):
    // the partner g ^ 2 holds j0 + g (its t = 2) and j0 + (1 ^ g) (its t = 3); then g ^ 1 holds
    // j0 + g as its t = 1
    auto reduce4 = [&](const float* p) -> float {
      const float q0 = p[0] + __shfl_xor_sync(0xffffffffu, p[2], 16);
      const float q1 = p[1] + __shfl_xor_sync(0xffffffffu, p[3], 16);
      return q0 + __shfl_xor_sync(0xffffffffu, q1, 8);
    };
    // eight tokens c0 + s0 .. c0 + s0 + 7 from the staged rows (s0 = their position in the stage);
    // lane group g handles each group of four in the order (t ^ g)
    auto step = [&](int s0, int j0, bool tail) {
      // c[t] = this group's word of token s0 + (t & 4) + ((t & 3) ^ g): the XOR order as two
      // conditional pair swaps of the loaded words
      uint32_t c[8];
#pragma unroll
      for (int h = 0; h < 8; h += 4) {
        const Word4 w = stage_g[(s0 + h) / 4];
        uint32_t v[4] = {word_of(w, 0), word_of(w, 1), word_of(w, 2), word_of(w, 3)};
        if (g & 1) {
          const uint32_t t0 = v[0], t2 = v[2];
          v[0] = v[1]; v[1] = t0; v[2] = v[3]; v[3] = t2;
        }
        if (g & 2) {
          const uint32_t t0 = v[0], t1 = v[1];
          v[0] = v[2]; v[1] = v[3]; v[2] = t0; v[3] = t1;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) c[h + u] = v[u];
      }
      float p[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        float acc = lookup(0, row_off(c[t], 0));
#pragma unroll
        for (int aa = 1; aa < A; ++aa) acc += lookup(aa, row_off(c[t], aa));
        p[t] = acc;
      }
      const float s0v = reduce4(p), s1v = reduce4(p + 4);
      if (!tail) {
        run = fmax3(run, s0v, s1v);
      } else {
        if (j0 + g < len) run = fmaxf(run, s0v);
        if (j0 + 4 + g < len) run = fmaxf(run, s1v);
      }
    };
    if (len > 0) {
      CodeRow nxt = __ldg(rows + min(lane, last));
      for (int c0 = 0; c0 < len; c0 += 32) {
        const CodeRow cur = nxt;
        if (c0 + 32 < len) nxt = __ldg(rows + min(c0 + 32 + lane, last));
        __syncwarp();
#pragma unroll
        for (int gg = 0; gg < 4; ++gg) stage[gg * kStagePitch + lane] = row_word(cur, gg);
        __syncwarp();
        const int n = min(32, len - c0);
        if (n == 32) {
#pragma unroll
          for (int s0 = 0; s0 < 32; s0 += 8) step(s0, c0 + s0, false);
        } else {
          for (int s0 = 0; s0 < n; s0 += 8) step(s0, c0 + s0, s0 + 8 > n);
        }
      }
    }
    run = fmaxf(run, __shfl_xor_sync(0xffffffffu, run, 8));
    run = fmaxf(run, __shfl_xor_sync(0xffffffffu, run, 16));
    float tot = (i < ns) ? run : 0.0f;
    tot += __shfl_xor_sync(0xffffffffu, tot, 1);
    tot += __shfl_xor_sync(0xffffffffu, tot, 2);
    tot += __shfl_xor_sync(0xffffffffu, tot, 4);
    if (lane == 0) a.out[static_cast<int64_t>(slice_id) * n_docs + doc] = tot;
  }
}

__global__ void pq_sum_slices_kernel(const float* __restrict__ partial, float* __restrict__ out,
                                     int64_t n_queries, int64_t n_docs, int nslice) {
  const int64_t total = n_queries * n_docs;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t q = i / n_docs, dd = i - q * n_docs;
    float s = 0.0f;
    for (int p = 0; p < nslice; ++p) s += partial[(q * nslice + p) * n_docs + dd];
    out[i] = s;
  }
}

int pick_qs(int64_t M, int64_t K, int64_t nq) {
  int qs = 8;
  while (qs > 1 && M * K * qs * 4 > kPqTableBudget) qs >>= 1;
  while (qs > 1 && qs / 2 >= nq) qs >>= 1;  // no wider than the query
  return qs;
}

template <int QS>
int launch_pq_t(const PqArgs& a, bool m16, unsigned grid, size_t smem, cudaStream_t st) {
  auto k = m16 ? pq_maxsim_kernel<QS, true> : pq_maxsim_kernel<QS, false>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return TMS_ERR_CUDA;
  k<<<grid, kPqThreads, smem, st>>>(a);
  return cuda_status(cudaGetLastError());
}

}  // namespace
}  // namespace tms

using namespace tms;

extern "C" int tms_pq_table(const void* Q, int q_dtype, int64_t n_queries, int64_t nq,
                            const void* codebook, int cb_dtype, int64_t M, int64_t K, int64_t dsub,
                            float* table, void* stream) {
  NvtxRange nvtx_range("tms_pq_table");
  if (n_queries < 0 || nq < 0 || M <= 0 || K <= 0 || dsub <= 0) return TMS_ERR_INVALID;
  if (q_dtype < TMS_F16 || q_dtype > TMS_F32 || cb_dtype < TMS_F16 || cb_dtype > TMS_F32)
    return TMS_ERR_INVALID;
  if (n_queries * nq == 0) return TMS_OK;
  if (!Q || !codebook || !table) return TMS_ERR_INVALID;
  int status = TMS_OK;
  const DeviceInfo* dev = current_device_info(&status);
  if (!dev) return status;
  const int64_t total = n_queries * nq * M * K;
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > dev->num_sms * 16) blocks = dev->num_sms * 16;
  pq_table_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      Q, q_dtype, n_queries * nq, codebook, cb_dtype, static_cast<int>(M), static_cast<int>(K),
      static_cast<int>(dsub), table);
  return cuda_status(cudaGetLastError());
}

namespace {
size_t pq_lut_workspace_size(int64_t n_queries, int64_t nq, int64_t M, int64_t K, int64_t n_docs) {
  const int qs = pick_qs(M, K, nq);
  const int64_t nslice = (nq + qs - 1) / qs;
  return nslice > 1 ? static_cast<size_t>(n_queries * nslice * n_docs) * 4 : 0;
}
// Both paths need at most this much (the tensor-core path's packed query tiles + partials, or the
// table-lookup path's per-slice partial scores).
size_t pq_ws_bytes(int64_t n_queries, int64_t nq, int64_t M, int64_t K, int64_t dsub,
                   int64_t n_docs) {
  size_t w = pq_lut_workspace_size(n_queries, nq, M, K, n_docs);
  if (pq_mma_codebook_bytes(M, K, dsub)) {
    const size_t m = pq_mma_workspace_size(n_queries, nq, M * dsub, n_docs);
    if (m > w) w = m;
  }
  return w;
}
}  // namespace

extern "C" size_t tms_pq_workspace_size(int64_t n_queries, int64_t nq, int64_t M, int64_t K,
                                        int64_t dsub, int64_t n_docs) {
  if (n_queries <= 0 || nq <= 0 || M <= 0 || K <= 0 || dsub <= 0 || n_docs < 0) return 0;
  return pq_ws_bytes(n_queries, nq, M, K, dsub, n_docs);
}

extern "C" int tms_pq_maxsim(const void* Q, int q_dtype, int64_t n_queries, int64_t nq,
                             const void* codebook, int cb_dtype, int64_t M, int64_t K,
                             int64_t dsub, const uint8_t* codes, int64_t n_tokens,
                             const int64_t* doc_offsets, int64_t n_docs, int64_t nd_uniform,
                             float* out, int mode, void* workspace, size_t workspace_bytes,
                             void* stream) {
  NvtxRange nvtx_range("tms_pq_maxsim");
  if (mode != TMS_PQ_FAST && mode != TMS_PQ_EXACT && mode != TMS_PQ_PRECISE) return TMS_ERR_INVALID;
  if (n_queries < 0 || nq <= 0 || M <= 0 || K <= 0 || dsub <= 0 || n_docs < 0 || n_tokens < 0)
    return TMS_ERR_INVALID;
  if (q_dtype < TMS_F16 || q_dtype > TMS_F32 || cb_dtype < TMS_F16 || cb_dtype > TMS_F32)
    return TMS_ERR_INVALID;
  if (n_queries == 0 || n_docs == 0) return TMS_OK;
  if (K > 256 || M > 4096) return TMS_ERR_UNSUPPORTED;  // codes are bytes
  if (!Q || !codebook || !out || (n_tokens > 0 && !codes)) return TMS_ERR_INVALID;
  if (!doc_offsets && (nd_uniform < 0 || n_docs * nd_uniform > n_tokens)) return TMS_ERR_INVALID;
  int status = TMS_OK;
  const DeviceInfo* dev = current_device_info(&status);
  if (!dev) return status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // TMS_PQ_PRECISE with fp16 queries of up to 128 rows: the token-rows tensor kernel with the
  // codebook split into fp16 hi + lo (the reference's precision), in passes of up to four 32-row
  // query chunks (four queries of <= 32 tokens, two of <= 64, one of <= 128). A pass decodes the
  // corpus once for its queries, while the table lookups below cost ceil(Nq / 8) table slices per
  // query, so batches of queries with <= 8 tokens that need more than one pass keep the lookups.
  const int64_t nchunk_q = (nq + 31) / 32;
  if (mode == TMS_PQ_PRECISE && q_dtype == TMS_F16 && nchunk_q <= 4 &&
      (n_queries * nchunk_q <= 4 || nq >= 9)) {
    const int64_t per = 4 / nchunk_q;  // queries per pass
    const int64_t d = M * dsub;
    int rc = TMS_OK;
    for (int64_t q0 = 0; q0 < n_queries && rc == TMS_OK; q0 += per) {
      const int64_t nqry = n_queries - q0 < per ? n_queries - q0 : per;
      // every pass has the same shape: only the first can answer TMS_ERR_UNSUPPORTED
      rc = pq_tokrows_maxsim(static_cast<const __half*>(Q) + q0 * nq * d, nqry, nq, codebook,
                             cb_dtype, M, K, dsub, codes, n_tokens, doc_offsets, n_docs,
                             nd_uniform, out + q0 * n_docs, workspace, workspace_bytes, st, true);
    }
    if (rc != TMS_ERR_UNSUPPORTED) return rc;
  }
  // Tensor-core path: codes decoded through a shared-memory fp16 codebook into MMA operand tiles
  // (fp16 queries, TMS_PQ_FAST); otherwise the exact fp32 table-lookup kernel below.
  if (mode == TMS_PQ_FAST && q_dtype == TMS_F16 && pq_mma_codebook_bytes(M, K, dsub)) {
    // up to four 32-row query chunks: decoded tokens as the TMEM A operand (pq_tokrows.cu); more
    // chunks go to the dense kernel's decoder warps (one decode for the whole batch)
    {
      const int rc = pq_tokrows_maxsim(Q, n_queries, nq, codebook, cb_dtype, M, K, dsub, codes,
                                       n_tokens, doc_offsets, n_docs, nd_uniform, out, workspace,
                                       workspace_bytes, st, false);
      if (rc != TMS_ERR_UNSUPPORTED) return rc;
    }
    const int rc = pq_mma_maxsim(Q, n_queries, nq, codebook, cb_dtype, M, K, dsub, codes, n_tokens,
                                 doc_offsets, n_docs, nd_uniform, out, workspace, workspace_bytes,
                                 st);
    if (rc != TMS_ERR_UNSUPPORTED) return rc;
  }
  // conflict-free lookups for M = 8 / 16 (code rows aligned to their size), else the general kernel
  const bool lut4 = (M == 16 || M == 8) && (reinterpret_cast<uintptr_t>(codes) % M) == 0 &&
                    M * K * 32 <= kPqTableBudget;
  const int qs = lut4 ? 8 : pick_qs(M, K, nq);
  // lut4: the table plus one 32-row code stage per warp
  const size_t smem = lut4 ? static_cast<size_t>(M * K * 32) + (kLut4Threads / 32) * 4 * 144
                           : static_cast<size_t>(M * K * qs) * 4;
  if (static_cast<int>(smem) > dev->max_smem_optin) return TMS_ERR_UNSUPPORTED;
  const int nslice = static_cast<int>((nq + qs - 1) / qs);
  const size_t need = nslice > 1 ? static_cast<size_t>(n_queries * nslice * n_docs) * 4 : 0;
  if (need && (!workspace || workspace_bytes < need)) return TMS_ERR_WORKSPACE;
  const bool m16 = (M == 16) && ((reinterpret_cast<uintptr_t>(codes) & 15) == 0);

  PqArgs a;
  a.Q = Q;
  a.cb = codebook;
  a.codes = codes;
  a.n_tokens = n_tokens;
  a.docs.offsets = doc_offsets;
  a.docs.n_docs = n_docs;
  a.docs.nd = doc_offsets ? 0 : nd_uniform;
  a.out = nslice > 1 ? static_cast<float*>(workspace) : out;
  a.q_dtype = q_dtype;
  a.cb_dtype = cb_dtype;
  a.nq = static_cast<int>(nq);
  a.M = static_cast<int>(M);
  a.K = static_cast<int>(K);
  a.dsub = static_cast<int>(dsub);
  a.nslice = nslice;
  const int64_t slices = n_queries * nslice;
  int64_t parts = (2LL * dev->num_sms + slices - 1) / slices;
  if (lut4) {
    // one 512-thread CTA per SM: the fewest document parts that make slices x parts a whole
    // number of waves (gcd rule)
    int64_t gcd = dev->num_sms, gb = slices;
    while (gb) { const int64_t t = gcd % gb; gcd = gb; gb = t; }
    parts = dev->num_sms / gcd;
  }
  const int64_t max_parts = (n_docs + 15) / 16;  // at least ~16 docs per CTA
  if (parts > max_parts) parts = max_parts;
  if (parts < 1) parts = 1;
  if (slices * parts > 0x7fffffffLL) return TMS_ERR_UNSUPPORTED;
  a.n_doc_parts = static_cast<int>(parts);
  const unsigned grid = static_cast<unsigned>(slices * parts);
  int rc;
  if (lut4) {
    auto k = (M == 16) ? (K == 256 ? pq_lut4_kernel<4, 256> : pq_lut4_kernel<4, 0>)
                       : (K == 256 ? pq_lut4_kernel<2, 256> : pq_lut4_kernel<2, 0>);
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return TMS_ERR_CUDA;
    k<<<grid, kLut4Threads, smem, st>>>(a);
    rc = cuda_status(cudaGetLastError());
  } else switch (qs) {
    case 8: rc = launch_pq_t<8>(a, m16, grid, smem, st); break;
    case 4: rc = launch_pq_t<4>(a, m16, grid, smem, st); break;
    case 2: rc = launch_pq_t<2>(a, m16, grid, smem, st); break;
    default: rc = launch_pq_t<1>(a, m16, grid, smem, st); break;
  }
  if (rc != TMS_OK || nslice == 1) return rc;
  const int64_t total = n_queries * n_docs;
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > dev->num_sms * 8) blocks = dev->num_sms * 8;
  pq_sum_slices_kernel<<<blocks, 256, 0, st>>>(static_cast<const float*>(workspace), out,
                                               n_queries, n_docs, nslice);
  return cuda_status(cudaGetLastError());
}
