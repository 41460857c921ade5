// jb_encode_text_device_noalloc: the text encoder forward of
// jb_encode_text_device for callers that must not allocate device memory.
//
// Who cannot allocate, and why: cudaMalloc and cudaFree synchronise the whole
// device, so a latency-critical caller (single-row query encoding running
// beside a bulk embedding job on the same GPU) would stall behind the bulk
// job's kernels the first time a workspace has to grow; and a caller whose
// device memory is fully reserved by another runtime's pool (a serving
// process that pre-reserves most of HBM) has nothing left to cudaMalloc
// from.  This entry point uses no cudaMalloc, cudaFree or allocating library
// routine: its working memory is the file-scope array below, which exists on
// every GPU that loads the library until the process exits.
//
// Limits and sharing:
//  * at most kNoAllocScratchBytes (64 MiB) of workspace per call, i.e.
//    jb_estimate_batch_bytes(model, batch, max_seq) <= 64 MiB (about 3,000
//    token slots of batch x max_seq for a 768-wide bf16 BERT); larger calls
//    are rejected with JB_ERR_INVALID before any work is queued;
//  * every call on a device shares the one array, and it keeps the previous
//    call's contents: calls that overlap on the GPU (concurrent streams,
//    other handles on the same device) race and must be serialised by the
//    caller.  Nothing in it needs to start at zero: every value a call reads
//    is written earlier in the same call (rows past the live token count feed
//    only discarded tile rows of the GEMMs);
//  * the first call on a device resolves the array's device address
//    (cudaGetSymbolAddress, with that device current); make that first call
//    before any stream capture.  Nothing else is set up on a call: the int8
//    GELU table (also a file-scope device array) is built when an int8 model
//    loads.  The cached address is not valid after cudaDeviceReset, which
//    also invalidates every model handle on that device;
//  * device-side input errors (an id outside the vocabulary, a length above
//    max_seq) are flagged on the device and reported by the handle's next
//    synchronising call, as for jb_encode_text_device.
#include <mutex>

#include "jb_model.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device.  In host code the symbol
// is only a host-side stand-in, never a device address.
std::mutex g_addr_mu;
void* g_addr[64] = {nullptr};

void* scratch_address(int device) {
  if (device < 0 || device >= 64) jb::fail(JB_ERR_INVALID, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_addr_mu);
  if (!g_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // device is current
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      jb::fail(JB_ERR_CUDA, std::string("cudaGetSymbolAddress(no-alloc scratch): ") +
                                cudaGetErrorString(e));
    }
    g_addr[device] = p;
  }
  return g_addr[device];
}

// Points the handle at the static scratch (and pauses event profiling, whose
// events would be created on demand) for the duration of one call.
struct ScratchOverride {
  jb_model* m;
  jb::Workspace saved;
  bool prof;
  ScratchOverride(jb_model* m_, const jb::Workspace& ws) : m(m_), saved(m_->ws), prof(m_->prof_on) {
    m->ws = ws;
    m->prof_on = false;
  }
  ~ScratchOverride() {
    m->ws = saved;
    m->prof_on = prof;
  }
};

}  // namespace

extern "C" jb_status jb_encode_text_device_noalloc(jb_model* m, const uint32_t* d_ids,
                                                   const uint32_t* d_lens, int batch, int max_seq,
                                                   int pooling, float* d_out, void* stream) {
  try {
    if (!m) jb::fail(JB_ERR_INVALID, "null model");
    if (m->family != JB_FAMILY_BERT)
      jb::fail(JB_ERR_INVALID, m->family == JB_FAMILY_CLIP_TEXT
                                   ? "jb_encode_text_device_noalloc serves BERT-family encoders only, "
                                     "not the OpenCLIP text tower"
                                   : "jb_encode_text_device_noalloc serves BERT-family text encoders "
                                     "only, not an image encoder");
    if (batch < 0 || max_seq < 0) jb::fail(JB_ERR_INVALID, "batch and max_seq must be >= 0");
    if (pooling < JB_POOL_MEAN || pooling > JB_POOL_WEIGHTED_MEAN) jb::fail(JB_ERR_INVALID, "unknown pooling");
    if (max_seq > m->max_pos)
      jb::fail(JB_ERR_SEQ_TOO_LONG, "sequence length " + std::to_string(max_seq) +
                                        " exceeds max_position_embeddings " + std::to_string(m->max_pos));
    if (batch > 0) {
      if (!d_ids || !d_lens || !d_out) jb::fail(JB_ERR_INVALID, "null buffer");
      const int seq = max_seq > 0 ? max_seq : 1;
      const size_t need = jb::estimate_batch_bytes(m, batch, seq);
      if (need > kNoAllocScratchBytes)
        jb::fail(JB_ERR_INVALID, "jb_encode_text_device_noalloc: batch " + std::to_string(batch) +
                                     " x seq " + std::to_string(seq) + " needs " + std::to_string(need) +
                                     " bytes of scratch; the limit is " +
                                     std::to_string(kNoAllocScratchBytes) + " bytes (64 MiB)");
      std::lock_guard<std::mutex> lk(m->mu);
      jb::DeviceGuard g(m->device);
      ScratchOverride ov(m, jb::carve_workspace(m, scratch_address(m->device), batch, seq));
      jb::bert_forward_device(m, d_ids, d_lens, batch, max_seq, pooling, d_out, nullptr,
                              reinterpret_cast<cudaStream_t>(stream));
    }
    return jb::record_error(JB_OK, "");
  } catch (const jb::Error& e) {
    return jb::record_error(e.status, e.msg);
  } catch (const std::exception& e) {
    return jb::record_error(JB_ERR_INVALID, e.what());
  }
}
