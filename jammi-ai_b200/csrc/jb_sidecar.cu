// The ANN sidecar's insert and search on the device: the embeddings a job
// produces go into the sidecar's vector store without a host loop per row.
//
// * add (ResultSink::write_batch, crates/jammi-ai/src/pipeline/
//   result_sink.rs:61-83, which keeps the rows whose status is ok and feeds
//   each to SidecarIndex::add, crates/jammi-db/src/index/sidecar.rs:754-790):
//   the rows of a batch whose validity bit is set are appended in row order,
//   each taking the next internal key, into the exact-f32 store -- the
//   buffer the reference accumulates for its .rawf32 rescore companion.  One
//   kernel per chunk of rows: each CTA counts the valid rows before its 256
//   from the bitmap, ballots its own, and its warps copy the valid rows to
//   their keys with 16-byte loads and stores.
// * build (SidecarIndex::build, sidecar.rs:792-824): for a Binary sidecar
//   the per-dimension threshold tau is fit over the store (fit_binary_
//   threshold, sidecar.rs:162-216) and every row sign-packed against it
//   (pack_threshold_bits, sidecar.rs:232-241) -- the codes the reference
//   inserts into its usearch b1x8 graph, one per key.
// * search (SidecarIndex::search, sidecar.rs:826-864): Binary -- the query
//   packed against the same tau, Hamming distance (differing bits) to every
//   code, the k nearest under (distance, tie rank); F32 -- cosine distance
//   (crates/jammi-numerics/src/distance.rs:6-21) to every stored vector.
//   The reference walks an HNSW graph (usearch, a third-party library) and
//   returns approximate neighbours; this scans every key and returns the
//   exact ones, which is what a graph of perfect recall returns.
// * search_final (SegmentedIndex::search_final, crates/jammi-db/src/index/
//   segment.rs:239-264): retrieve k x oversample candidates (at least k) by
//   search, rescore each with the exact cosine distance to its stored f32
//   vector, order by (distance under f32 total order, tie rank), keep k.
//
// Ties: the reference orders equal distances by _row_id; the caller passes
// each key's rank in ascending _row_id order to build (NULL = key order).
#include <cfloat>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>

#include "jb_model.h"

struct jb_sidecar {
  int device = 0;
  int dim = 0;
  int nb = 0;  // code bytes per row, ceil(dim / 8)
  int precision = JB_STORAGE_F32;
  int64_t len = 0;
  bool built = false;
  int threshold_kind = -1;
  bool has_rank = false;
  cudaStream_t stream = nullptr;
  std::mutex mu;
  // device buffers and their capacities in bytes
  float* exact = nullptr;
  size_t exact_cap = 0;
  uint8_t* codes = nullptr;
  size_t codes_cap = 0;
  float* tau = nullptr;
  unsigned char* fit = nullptr;  // threshold fit scratch
  size_t fit_cap = 0;
  uint32_t* rank = nullptr;
  size_t rank_cap = 0;
  float* in = nullptr;  // add staging
  size_t in_cap = 0;
  uint8_t* valid = nullptr;
  size_t valid_cap = 0;
  float* q = nullptr;  // search staging
  size_t q_cap = 0;
  uint8_t* qcodes = nullptr;
  size_t qcodes_cap = 0;
  float* scratch = nullptr;
  size_t scratch_cap = 0;
  int64_t* cand = nullptr;
  size_t cand_cap = 0;
  float* cand_dist = nullptr;
  size_t cand_dist_cap = 0;
  float* resc = nullptr;
  size_t resc_cap = 0;
  int64_t* out_idx = nullptr;
  size_t out_idx_cap = 0;
  float* out_dist = nullptr;
  size_t out_dist_cap = 0;
  int64_t* d_len = nullptr;  // [0] keys before the chunk, [1] running total
  int* err = nullptr;
};

namespace {

constexpr int kCompactRows = 256;
constexpr int kHamRows = 256;
constexpr int kHamQ = 8;
constexpr int kHamWords = 16;
constexpr size_t kAddChunkBytes = size_t(64) << 20;    // staging per add chunk
constexpr int64_t kAddChunkRows = 131072;               // and at most this many rows
constexpr size_t kScratchBytes = size_t(256) << 20;   // distance matrix per query batch

__device__ __forceinline__ uint32_t total_key(float x) {
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__global__ void set_len_kernel(int64_t* d_len, int64_t len) {
  d_len[0] = len;
  d_len[1] = len;
}
__global__ void commit_len_kernel(int64_t* d_len) { d_len[0] = d_len[1]; }

// Rows [0, nr) of in [nr, dim]: the valid ones (bit r of valid, LSB-first;
// NULL = all) go to store rows d_len[0] + (valid rows before r), in order.
template <bool kVec4>
__global__ void __launch_bounds__(kCompactRows)
compact_rows_kernel(const float* __restrict__ in, int nr, int dim, const uint8_t* __restrict__ valid,
                    float* __restrict__ store, int64_t* d_len) {
  __shared__ int s_before[kCompactRows / 32];
  __shared__ int s_warp[kCompactRows / 32];
  __shared__ int s_pos[kCompactRows];
  __shared__ int64_t s_base;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int r0 = blockIdx.x * kCompactRows;  // a multiple of 8: whole bitmap bytes before it
  int before = 0;
  if (valid) {
    for (int i = t; i < r0 / 8; i += kCompactRows) before += __popc(static_cast<unsigned>(valid[i]));
  } else if (t == 0) {
    before = r0;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) before += __shfl_xor_sync(0xFFFFFFFFu, before, o);
  const int r = r0 + t;
  const bool v = r < nr && (valid == nullptr || ((valid[r >> 3] >> (r & 7)) & 1));
  const unsigned bal = __ballot_sync(0xFFFFFFFFu, v);
  if (lane == 0) {
    s_before[w] = before;
    s_warp[w] = __popc(bal);
  }
  __syncthreads();
  int pos = __popc(bal & ((1u << lane) - 1u));
  for (int i = 0; i < w; ++i) pos += s_warp[i];
  s_pos[t] = v ? pos : -1;
  if (t == 0) {
    int64_t b = d_len[0];
    int cnt = 0;
    for (int i = 0; i < kCompactRows / 32; ++i) {
      b += s_before[i];
      cnt += s_warp[i];
    }
    s_base = b;
    atomicAdd(reinterpret_cast<unsigned long long*>(d_len + 1), static_cast<unsigned long long>(cnt));
  }
  __syncthreads();
  const int64_t base = s_base;
  for (int j = w; j < kCompactRows; j += kCompactRows / 32) {
    const int p = s_pos[j];
    if (p < 0) continue;
    const float* src = in + static_cast<int64_t>(r0 + j) * dim;
    float* dst = store + (base + p) * dim;
    if (kVec4) {  // four 16-byte loads in flight per lane
      const float4* s4 = reinterpret_cast<const float4*>(src);
      float4* d4 = reinterpret_cast<float4*>(dst);
      const int n4 = dim / 4;
      for (int c0 = lane; c0 < n4; c0 += 32 * 4) {
        float4 t4[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (c0 + 32 * u < n4) t4[u] = __ldg(s4 + c0 + 32 * u);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (c0 + 32 * u < n4) d4[c0 + 32 * u] = t4[u];
      }
    } else {
      for (int c = lane; c < dim; c += 32) dst[c] = __ldg(src + c);
    }
  }
}

// Word w (bytes 4w .. 4w+3, little-endian) of a code row of nb bytes; bytes
// past nb read as 0.
template <bool kAligned>
__device__ __forceinline__ uint32_t code_word(const uint8_t* row, int nb, int w) {
  if (kAligned) return __ldg(reinterpret_cast<const uint32_t*>(row) + w);
  uint32_t x = 0;
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const int i = 4 * w + b;
    if (i < nb) x |= static_cast<uint32_t>(__ldg(row + i)) << (8 * b);
  }
  return x;
}

// dist[q][row] = differing bits of query code q and code row, as f32, for
// queries [q0, q0 + 8) x rows [row0, row0 + 256).
template <bool kAligned>
__global__ void __launch_bounds__(kHamRows, 1)
hamming_kernel(const uint8_t* __restrict__ codes, int64_t n, int nb, const uint8_t* __restrict__ qcodes,
               int nq, float* __restrict__ dist) {
  __shared__ uint32_t tile[kHamRows][kHamWords + 1];
  __shared__ uint32_t qs[kHamQ][kHamWords];
  const int t = threadIdx.x;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kHamRows;
  const int q0 = blockIdx.y * kHamQ;
  const int nw = (nb + 3) / 4;
  int cnt[kHamQ];
#pragma unroll
  for (int j = 0; j < kHamQ; ++j) cnt[j] = 0;
  for (int w0 = 0; w0 < nw; w0 += kHamWords) {
    const int ww = min(kHamWords, nw - w0);
#pragma unroll 4
    for (int e = t; e < kHamRows * kHamWords; e += kHamRows) {
      const int r = e / kHamWords, c = e % kHamWords;
      const int64_t gr = row0 + r;
      tile[r][c] = (gr < n && c < ww) ? code_word<kAligned>(codes + gr * nb, nb, w0 + c) : 0u;
    }
    for (int e = t; e < kHamQ * kHamWords; e += kHamRows) {
      const int j = e / kHamWords, c = e % kHamWords;
      qs[j][c] = (q0 + j < nq && c < ww)
                     ? code_word<kAligned>(qcodes + static_cast<int64_t>(q0 + j) * nb, nb, w0 + c)
                     : 0u;
    }
    __syncthreads();
    for (int c = 0; c < ww; ++c) {
      const uint32_t x = tile[t][c];
#pragma unroll
      for (int j = 0; j < kHamQ; ++j) cnt[j] += __popc(x ^ qs[j][c]);
    }
    __syncthreads();
  }
  const int64_t row = row0 + t;
  if (row >= n) return;
#pragma unroll
  for (int j = 0; j < kHamQ; ++j)
    if (q0 + j < nq) dist[static_cast<int64_t>(q0 + j) * n + row] = static_cast<float>(cnt[j]);
}

// out[q][j] = cosine_distance(query q, store row cand[q][j]) in the
// reference's f32 operation order (each product and sum rounded, dimension
// order, no fused multiply-add); +inf for an empty slot (cand < 0).
__global__ void rescore_kernel(const float* __restrict__ store, int dim, const float* __restrict__ q,
                               int nq, const int64_t* __restrict__ cand, int ck, float* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(nq) * ck) return;
  const int64_t key = cand[i];
  if (key < 0) {
    out[i] = __uint_as_float(0x7F800000u);
    return;
  }
  const float* a = q + (i / ck) * dim;
  const float* b = store + key * dim;
  float dot = 0.0f, na = 0.0f, nb = 0.0f;
  for (int d = 0; d < dim; ++d) {
    const float x = __ldg(a + d), y = __ldg(b + d);
    dot = __fadd_rn(dot, __fmul_rn(x, y));
    na = __fadd_rn(na, __fmul_rn(x, x));
    nb = __fadd_rn(nb, __fmul_rn(y, y));
  }
  const float denom = __fmul_rn(__fsqrt_rn(na), __fsqrt_rn(nb));
  out[i] = denom < FLT_EPSILON ? 1.0f : __fsub_rn(1.0f, __fdiv_rn(dot, denom));
}

// One CTA per query: the ck rescored candidates ordered by (distance under
// f32 total order -- f32::total_cmp --, tie rank); the first k written,
// slots past ck -1 / +inf.
__global__ void __launch_bounds__(jb::kMaxSearchK)
rescore_order_kernel(const float* __restrict__ resc, const int64_t* __restrict__ cand, int ck,
                     const uint32_t* __restrict__ rank, int k, int64_t* __restrict__ out_idx,
                     float* __restrict__ out_dist) {
  __shared__ uint64_t key[jb::kMaxSearchK];
  const int q = blockIdx.x, t = threadIdx.x;
  for (int s = ck + t; s < k; s += blockDim.x) {
    out_idx[static_cast<int64_t>(q) * k + s] = -1;
    out_dist[static_cast<int64_t>(q) * k + s] = __uint_as_float(0x7F800000u);
  }
  int64_t c = -1;
  float d = 0.0f;
  if (t < ck) {
    c = cand[static_cast<int64_t>(q) * ck + t];
    d = resc[static_cast<int64_t>(q) * ck + t];
    const uint32_t rk = c < 0 ? 0xFFFFFFFFu : (rank ? rank[c] : static_cast<uint32_t>(c));
    key[t] = (static_cast<uint64_t>(total_key(d)) << 32) | rk;
  }
  __syncthreads();
  if (t >= ck) return;
  const uint64_t mine = key[t];
  int pos = 0;
  for (int j = 0; j < ck; ++j) pos += key[j] < mine || (key[j] == mine && j < t);
  if (pos < k) {
    out_idx[static_cast<int64_t>(q) * k + pos] = c;
    out_dist[static_cast<int64_t>(q) * k + pos] = d;
  }
}

// ---- host side --------------------------------------------------------------

template <typename T>
void ensure(T** p, size_t* cap, size_t bytes, bool keep, cudaStream_t s) {
  if (bytes <= *cap) return;
  size_t want = *cap * 2 > bytes ? *cap * 2 : bytes;
  want = (want + 255) & ~size_t(255);
  T* np = nullptr;
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&np), want);
  if (e == cudaErrorMemoryAllocation && want > bytes) {  // doubling did not fit: the exact size
    cudaGetLastError();
    want = (bytes + 255) & ~size_t(255);
    e = cudaMalloc(reinterpret_cast<void**>(&np), want);
  }
  jb::check_cuda(e, "sidecar buffer");
  if (keep && *p && *cap) {
    jb::check_cuda(cudaMemcpyAsync(np, *p, *cap, cudaMemcpyDeviceToDevice, s), "sidecar buffer copy");
    jb::check_cuda(cudaStreamSynchronize(s), "sidecar buffer copy");
  }
  if (*p) cudaFree(*p);
  *p = np;
  *cap = want;
}

void sync_and_check(jb_sidecar* x, const char* what) {
  jb::check_cuda(cudaStreamSynchronize(x->stream), what);
  int flag = 0;
  jb::check_cuda(cudaMemcpy(&flag, x->err, sizeof(int), cudaMemcpyDeviceToHost), what);
  if (flag) {
    jb::check_cuda(cudaMemset(x->err, 0, sizeof(int)), what);
    jb::fail(JB_ERR_INVALID, std::string(what) + ": repeated tie ranks (each key needs its own rank)");
  }
}

template <typename F>
jb_status guarded(F&& f) {
  try {
    f();
    return jb::record_error(JB_OK, "");
  } catch (const jb::Error& e) {
    return jb::record_error(e.status, e.msg);
  } catch (const std::bad_alloc&) {
    return jb::record_error(JB_ERR_OOM, "host out of memory");
  } catch (const std::exception& e) {
    return jb::record_error(JB_ERR_INVALID, e.what());
  }
}

void check_queries(const jb_sidecar* x, const float* queries, int nq, int k, int64_t* keys, float* dist,
                   const char* who) {
  if (!x) jb::fail(JB_ERR_INVALID, std::string(who) + ": null sidecar");
  if (nq < 0 || k < 0) jb::fail(JB_ERR_INVALID, std::string(who) + ": negative count");
  if (k > jb::kMaxSearchK)
    jb::fail(JB_ERR_INVALID, std::string(who) + ": k above " + std::to_string(jb::kMaxSearchK));
  if (nq > 0 && k > 0 && (!queries || !keys || !dist)) jb::fail(JB_ERR_INVALID, std::string(who) + ": null buffer");
}

// Fills keys / dist of queries [q0, q0 + nq) with -1 / +inf.
void fill_empty(int64_t* keys, float* dist, int64_t count) {
  const float inf = __builtin_huge_valf();
  for (int64_t i = 0; i < count; ++i) {
    keys[i] = -1;
    dist[i] = inf;
  }
}

// Memory of `device` itself (or managed memory): kernels there read it in place.
bool device_resident(const void* p, int device) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return (a.type == cudaMemoryTypeDevice && a.device == device) || a.type == cudaMemoryTypeManaged;
}

bool host_memory(const void* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return true;
  }
  return a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged;
}

// The k nearest keys of queries (any memory) [nq, dim] under the sidecar's
// own metric, k <= kMaxSearchK, into device out_idx / out_dist [nq, k].
// Queries are staged in x->q.
void search_device(jb_sidecar* x, const float* queries, int nq, int k, int64_t* out_idx, float* out_dist,
                   int64_t q_off) {
  cudaStream_t s = x->stream;
  const int64_t n = x->len;
  const uint32_t* rank = x->has_rank ? x->rank : nullptr;
  jb::check_cuda(cudaMemcpyAsync(x->q, queries + q_off * x->dim, size_t(nq) * x->dim * sizeof(float),
                                 cudaMemcpyDefault, s),
                 "sidecar queries");
  ensure(&x->scratch, &x->scratch_cap, size_t(nq) * size_t(n) * sizeof(float), false, s);
  if (n == 0) {  // no keys: every slot -1 / +inf
    jb::check_cuda(jb::launch_topk(x->scratch, 0, nullptr, nq, k, out_idx, out_dist, x->err, s), "sidecar top-k");
  } else if (x->precision == JB_STORAGE_BINARY) {
    jb::check_cuda(jb::launch_pack_threshold_bits(x->q, nq, x->dim, x->tau, x->qcodes, s), "sidecar query codes");
    const dim3 grid(static_cast<unsigned>((n + kHamRows - 1) / kHamRows), (nq + kHamQ - 1) / kHamQ);
    if (x->nb % 4 == 0)
      hamming_kernel<true><<<grid, kHamRows, 0, s>>>(x->codes, n, x->nb, x->qcodes, nq, x->scratch);
    else
      hamming_kernel<false><<<grid, kHamRows, 0, s>>>(x->codes, n, x->nb, x->qcodes, nq, x->scratch);
    jb::check_cuda(cudaGetLastError(), "sidecar hamming distances");
    jb::check_cuda(jb::launch_topk(x->scratch, n, rank, nq, k, out_idx, out_dist, x->err, s), "sidecar top-k");
  } else {
    jb::check_cuda(jb::launch_exact_search(x->exact, n, x->dim, rank, x->q, nq, k, x->scratch, out_idx, out_dist,
                                           x->err, s),
                   "sidecar cosine search");
  }
}

// Queries per batch so that the [batch, len] distance matrix stays within
// kScratchBytes (at least 1) and the launch grids within their limits.
int query_batch(const jb_sidecar* x) {
  const int64_t per = x->len > 0 ? x->len * int64_t(sizeof(float)) : 1;
  int64_t b = int64_t(kScratchBytes) / per;
  if (b < 1) b = 1;
  if (b > 4096) b = 4096;
  return static_cast<int>(b);
}

void stage_queries(jb_sidecar* x, int nqb) {
  ensure(&x->q, &x->q_cap, size_t(nqb) * x->dim * sizeof(float), false, x->stream);
  ensure(&x->qcodes, &x->qcodes_cap, size_t(nqb) * x->nb, false, x->stream);
}

}  // namespace

extern "C" {

jb_status jb_sidecar_create(int device, int dim, int precision, jb_sidecar** out) {
  return guarded([&] {
    if (!out) jb::fail(JB_ERR_INVALID, "jb_sidecar_create: null out");
    *out = nullptr;
    if (dim <= 0) jb::fail(JB_ERR_INVALID, "jb_sidecar_create: dimensions must be positive");
    if (precision != JB_STORAGE_F32 && precision != JB_STORAGE_BINARY)
      jb::fail(JB_ERR_INVALID,
               "jb_sidecar_create: precision must be JB_STORAGE_F32 or JB_STORAGE_BINARY (f16 and int8 "
               "quantisation happen inside the graph library)");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
      cudaGetLastError();
      jb::fail(JB_ERR_NO_DEVICE, "no CUDA device available (require_gpu)");
    }
    if (device < 0 || device >= ndev) jb::fail(JB_ERR_NO_DEVICE, "device ordinal out of range");
    jb::DeviceGuard g(device);
    jb_sidecar* x = new jb_sidecar();
    x->device = device;
    x->dim = dim;
    x->nb = (dim + 7) / 8;
    x->precision = precision;
    try {
      jb::check_cuda(cudaStreamCreateWithFlags(&x->stream, cudaStreamNonBlocking), "sidecar stream");
      jb::check_cuda(cudaMalloc(&x->d_len, 2 * sizeof(int64_t)), "sidecar counters");
      jb::check_cuda(cudaMalloc(&x->err, sizeof(int)), "sidecar error flag");
      jb::check_cuda(cudaMemset(x->err, 0, sizeof(int)), "sidecar error flag");
      jb::check_cuda(cudaMalloc(&x->tau, size_t(dim) * sizeof(float)), "sidecar threshold");
    } catch (...) {
      jb_sidecar_free(x);
      throw;
    }
    *out = x;
  });
}

jb_status jb_sidecar_add(jb_sidecar* x, const float* vectors, const uint8_t* validity, int64_t rows,
                         int64_t* first_key, int64_t* added) {
  return guarded([&] {
    if (!x) jb::fail(JB_ERR_INVALID, "jb_sidecar_add: null sidecar");
    if (rows < 0) jb::fail(JB_ERR_INVALID, "jb_sidecar_add: negative row count");
    if (rows > 0 && !vectors) jb::fail(JB_ERR_INVALID, "jb_sidecar_add: null vectors");
    std::lock_guard<std::mutex> lk(x->mu);
    jb::DeviceGuard g(x->device);
    if (first_key) *first_key = x->len;
    if (added) *added = 0;
    if (rows == 0) return;
    if (x->len + rows > int64_t(UINT32_MAX)) jb::fail(JB_ERR_INVALID, "jb_sidecar_add: more than 2^32 keys");
    cudaStream_t s = x->stream;
    const size_t row_bytes = size_t(x->dim) * sizeof(float);
    ensure(&x->exact, &x->exact_cap, size_t(x->len + rows) * row_bytes, true, s);
    // rows (and bitmap) already in this device's memory are read in place;
    // others are copied chunk by chunk into the staging buffers
    const bool direct = device_resident(vectors, x->device);
    const bool bits_direct = validity && device_resident(validity, x->device);
    // chunk: a multiple of 256 rows (whole bitmap bytes, whole CTAs)
    int64_t chunk = direct ? kAddChunkRows : int64_t(kAddChunkBytes / row_bytes) / kCompactRows * kCompactRows;
    if (chunk < kCompactRows) chunk = kCompactRows;
    if (chunk > kAddChunkRows) chunk = kAddChunkRows;  // each CTA rescans the bitmap before it
    if (chunk > rows) chunk = (rows + kCompactRows - 1) / kCompactRows * kCompactRows;
    if (!direct) ensure(&x->in, &x->in_cap, size_t(chunk) * row_bytes, false, s);
    if (validity && !bits_direct) ensure(&x->valid, &x->valid_cap, size_t(chunk / 8), false, s);
    set_len_kernel<<<1, 1, 0, s>>>(x->d_len, x->len);
    jb::check_cuda(cudaGetLastError(), "jb_sidecar_add");
    // 16-byte row access: a width of whole float4s and a 16-byte aligned base
    const bool vec4 = x->dim % 4 == 0 && (!direct || reinterpret_cast<uintptr_t>(vectors) % 16 == 0);
    for (int64_t r0 = 0; r0 < rows; r0 += chunk) {
      const int nr = static_cast<int>(rows - r0 < chunk ? rows - r0 : chunk);
      const float* src = vectors + r0 * x->dim;
      if (!direct) {
        jb::check_cuda(cudaMemcpyAsync(x->in, src, size_t(nr) * row_bytes, cudaMemcpyDefault, s),
                       "jb_sidecar_add: vectors");
        src = x->in;
      }
      const uint8_t* bits = nullptr;
      if (validity) {
        bits = validity + r0 / 8;
        if (!bits_direct) {
          jb::check_cuda(cudaMemcpyAsync(x->valid, bits, size_t(nr + 7) / 8, cudaMemcpyDefault, s),
                         "jb_sidecar_add: validity");
          bits = x->valid;
        }
      }
      const unsigned blocks = static_cast<unsigned>((nr + kCompactRows - 1) / kCompactRows);
      if (vec4)
        compact_rows_kernel<true><<<blocks, kCompactRows, 0, s>>>(src, nr, x->dim, bits, x->exact, x->d_len);
      else
        compact_rows_kernel<false><<<blocks, kCompactRows, 0, s>>>(src, nr, x->dim, bits, x->exact, x->d_len);
      commit_len_kernel<<<1, 1, 0, s>>>(x->d_len);
      jb::check_cuda(cudaGetLastError(), "jb_sidecar_add");
    }
    int64_t len = 0;
    jb::check_cuda(cudaMemcpyAsync(&len, x->d_len, sizeof(int64_t), cudaMemcpyDeviceToHost, s), "jb_sidecar_add");
    jb::check_cuda(cudaStreamSynchronize(s), "jb_sidecar_add");
    if (added) *added = len - x->len;
    if (len != x->len) {
      x->built = false;  // new keys have no codes (Binary) and no tie rank yet
      x->has_rank = false;
    }
    x->len = len;
  });
}

jb_status jb_sidecar_build(jb_sidecar* x, int threshold_kind, const uint32_t* tie_rank) {
  return guarded([&] {
    if (!x) jb::fail(JB_ERR_INVALID, "jb_sidecar_build: null sidecar");
    if (threshold_kind != JB_THRESHOLD_MEAN && threshold_kind != JB_THRESHOLD_MEDIAN)
      jb::fail(JB_ERR_INVALID, "jb_sidecar_build: unknown threshold kind");
    std::lock_guard<std::mutex> lk(x->mu);
    jb::DeviceGuard g(x->device);
    cudaStream_t s = x->stream;
    if (x->precision == JB_STORAGE_BINARY && x->len > 0) {
      ensure(&x->codes, &x->codes_cap, size_t(x->len) * x->nb, false, s);
      ensure(&x->fit, &x->fit_cap, jb::fit_threshold_scratch_bytes(x->dim), false, s);
      jb::check_cuda(jb::launch_fit_binary_threshold(x->exact, x->len, x->dim, threshold_kind, x->tau, x->fit, s),
                     "jb_sidecar_build: threshold");
      jb::check_cuda(jb::launch_pack_threshold_bits(x->exact, x->len, x->dim, x->tau, x->codes, s),
                     "jb_sidecar_build: codes");
      x->threshold_kind = threshold_kind;
    }
    x->has_rank = false;
    if (tie_rank && x->len > 0) {
      ensure(&x->rank, &x->rank_cap, size_t(x->len) * sizeof(uint32_t), false, s);
      jb::check_cuda(cudaMemcpyAsync(x->rank, tie_rank, size_t(x->len) * sizeof(uint32_t), cudaMemcpyDefault, s),
                     "jb_sidecar_build: tie ranks");
      x->has_rank = true;
    }
    jb::check_cuda(cudaStreamSynchronize(s), "jb_sidecar_build");
    x->built = true;
  });
}

int64_t jb_sidecar_len(const jb_sidecar* x) { return x ? x->len : -1; }

jb_status jb_sidecar_search(jb_sidecar* x, const float* queries, int n_queries, int k, int64_t* keys,
                            float* dist) {
  return guarded([&] {
    check_queries(x, queries, n_queries, k, keys, dist, "jb_sidecar_search");
    std::lock_guard<std::mutex> lk(x->mu);
    if (n_queries == 0 || k == 0) return;
    jb::DeviceGuard g(x->device);
    if (x->precision == JB_STORAGE_BINARY && x->len > 0 && !x->built)
      jb::fail(JB_ERR_INVALID, "Binary search: no threshold available -- the sidecar has not been built since "
                               "its last add");
    const bool host_out = host_memory(keys);
    if (x->len == 0) {
      if (host_out) {
        fill_empty(keys, dist, int64_t(n_queries) * k);
        return;
      }
    }
    cudaStream_t s = x->stream;
    const int qb = query_batch(x);
    stage_queries(x, qb);
    ensure(&x->out_idx, &x->out_idx_cap, size_t(qb) * k * sizeof(int64_t), false, s);
    ensure(&x->out_dist, &x->out_dist_cap, size_t(qb) * k * sizeof(float), false, s);
    for (int q0 = 0; q0 < n_queries; q0 += qb) {
      const int nq = n_queries - q0 < qb ? n_queries - q0 : qb;
      search_device(x, queries, nq, k, x->out_idx, x->out_dist, q0);
      jb::check_cuda(cudaMemcpyAsync(keys + int64_t(q0) * k, x->out_idx, size_t(nq) * k * sizeof(int64_t),
                                     cudaMemcpyDefault, s),
                     "jb_sidecar_search: keys");
      jb::check_cuda(cudaMemcpyAsync(dist + int64_t(q0) * k, x->out_dist, size_t(nq) * k * sizeof(float),
                                     cudaMemcpyDefault, s),
                     "jb_sidecar_search: distances");
      sync_and_check(x, "jb_sidecar_search");
    }
  });
}

jb_status jb_sidecar_search_final(jb_sidecar* x, const float* queries, int n_queries, int k, int oversample,
                                  int64_t* keys, float* dist) {
  if (x && x->precision == JB_STORAGE_F32)  // an exact store needs no rescore (segment.rs:245-247)
    return jb_sidecar_search(x, queries, n_queries, k, keys, dist);
  return guarded([&] {
    check_queries(x, queries, n_queries, k, keys, dist, "jb_sidecar_search_final");
    std::lock_guard<std::mutex> lk(x->mu);
    if (n_queries == 0 || k == 0) return;
    jb::DeviceGuard g(x->device);
    if (x->len > 0 && !x->built)
      jb::fail(JB_ERR_INVALID, "Binary search: no threshold available -- the sidecar has not been built since "
                               "its last add");
    // candidate_k = k x oversample, at least k (segment.rs:248); an
    // oversample below 1 counts as 1 (config.rs effective_oversample)
    const int64_t want = int64_t(k) * (oversample > 1 ? oversample : 1);
    if (want > jb::kMaxSearchK)
      jb::fail(JB_ERR_INVALID, "jb_sidecar_search_final: k x oversample = " + std::to_string(want) + " above " +
                                   std::to_string(jb::kMaxSearchK) + " candidates");
    const int ck = static_cast<int>(want < x->len ? want : x->len);
    const bool host_out = host_memory(keys);
    if (ck == 0 && host_out) {
      fill_empty(keys, dist, int64_t(n_queries) * k);
      return;
    }
    cudaStream_t s = x->stream;
    const int qb = query_batch(x);
    stage_queries(x, qb);
    ensure(&x->cand, &x->cand_cap, size_t(qb) * (ck > 0 ? ck : 1) * sizeof(int64_t), false, s);
    ensure(&x->cand_dist, &x->cand_dist_cap, size_t(qb) * (ck > 0 ? ck : 1) * sizeof(float), false, s);
    ensure(&x->resc, &x->resc_cap, size_t(qb) * (ck > 0 ? ck : 1) * sizeof(float), false, s);
    ensure(&x->out_idx, &x->out_idx_cap, size_t(qb) * k * sizeof(int64_t), false, s);
    ensure(&x->out_dist, &x->out_dist_cap, size_t(qb) * k * sizeof(float), false, s);
    const uint32_t* rank = x->has_rank ? x->rank : nullptr;
    for (int q0 = 0; q0 < n_queries; q0 += qb) {
      const int nq = n_queries - q0 < qb ? n_queries - q0 : qb;
      if (ck > 0) {
        search_device(x, queries, nq, ck, x->cand, x->cand_dist, q0);
        const int64_t pairs = int64_t(nq) * ck;
        rescore_kernel<<<static_cast<unsigned>((pairs + 127) / 128), 128, 0, s>>>(x->exact, x->dim, x->q, nq,
                                                                                 x->cand, ck, x->resc);
        jb::check_cuda(cudaGetLastError(), "jb_sidecar_search_final: rescore");
      }
      rescore_order_kernel<<<nq, jb::kMaxSearchK, 0, s>>>(x->resc, x->cand, ck, rank, k, x->out_idx, x->out_dist);
      jb::check_cuda(cudaGetLastError(), "jb_sidecar_search_final: order");
      jb::check_cuda(cudaMemcpyAsync(keys + int64_t(q0) * k, x->out_idx, size_t(nq) * k * sizeof(int64_t),
                                     cudaMemcpyDefault, s),
                     "jb_sidecar_search_final: keys");
      jb::check_cuda(cudaMemcpyAsync(dist + int64_t(q0) * k, x->out_dist, size_t(nq) * k * sizeof(float),
                                     cudaMemcpyDefault, s),
                     "jb_sidecar_search_final: distances");
      sync_and_check(x, "jb_sidecar_search_final");
    }
  });
}

jb_status jb_sidecar_export(jb_sidecar* x, float* exact, uint8_t* codes, float* tau) {
  return guarded([&] {
    if (!x) jb::fail(JB_ERR_INVALID, "jb_sidecar_export: null sidecar");
    std::lock_guard<std::mutex> lk(x->mu);
    jb::DeviceGuard g(x->device);
    const bool fitted = x->precision == JB_STORAGE_BINARY && x->built && x->len > 0;
    if ((codes || tau) && !fitted)
      jb::fail(JB_ERR_INVALID, "jb_sidecar_export: codes and threshold exist only for a built Binary sidecar "
                               "with at least one row");
    cudaStream_t s = x->stream;
    if (exact && x->len > 0)
      jb::check_cuda(cudaMemcpyAsync(exact, x->exact, size_t(x->len) * x->dim * sizeof(float), cudaMemcpyDefault, s),
                     "jb_sidecar_export: vectors");
    if (codes)
      jb::check_cuda(cudaMemcpyAsync(codes, x->codes, size_t(x->len) * x->nb, cudaMemcpyDefault, s),
                     "jb_sidecar_export: codes");
    if (tau)
      jb::check_cuda(cudaMemcpyAsync(tau, x->tau, size_t(x->dim) * sizeof(float), cudaMemcpyDefault, s),
                     "jb_sidecar_export: threshold");
    jb::check_cuda(cudaStreamSynchronize(s), "jb_sidecar_export");
  });
}

void jb_sidecar_free(jb_sidecar* x) {
  if (!x) return;
  int prev = -1;
  cudaGetDevice(&prev);
  if (cudaSetDevice(x->device) == cudaSuccess) {
    if (x->stream) cudaStreamSynchronize(x->stream);
    void* bufs[] = {x->exact, x->codes,     x->tau,  x->fit, x->rank,    x->in,       x->valid,  x->q,   x->qcodes,
                    x->scratch, x->cand, x->cand_dist, x->resc, x->out_idx, x->out_dist, x->d_len, x->err};
    for (void* p : bufs)
      if (p) cudaFree(p);
    if (x->stream) cudaStreamDestroy(x->stream);
  }
  cudaGetLastError();
  if (prev >= 0) cudaSetDevice(prev);
  delete x;
}

}  // extern "C"
