// ms_expert_mlp_static: the expert MLP of ms_expert_mlp for callers that are
// not allowed to allocate device memory.
//
// Some hosts cannot call cudaMalloc at the point where they run the expert
// block: an inference runtime that reserves all device memory up front and
// hands plugins only the buffers it planned, an engine whose enqueue step
// must never allocate, or a process that must not grow its footprint while
// serving. ms_expert_mlp needs a pool handle, and creating one allocates the
// slot arena and the scratch buffers. This entry point needs neither: the
// caller passes the expert weights (any device buffer laid out as n_slots
// blobs) plus the inputs and the output, and the intermediate buffers live in
// one file-scope __device__ array of fixed size, loaded with the library.
//
// Limits: T <= MS_STATIC_MAX_TOKENS tokens, T*k <= MS_STATIC_MAX_PAIRS,
// d_model and d_ff <= 4096 (3072 for gpt-oss), n_slots <= MS_STATIC_MAX_SLOTS. Every GPU that
// loads the library keeps the array (about 2 MB) until the process exits.
// All calls on a device share it, so two calls that can run at the same time
// on the GPU (different streams, different host threads) race and corrupt
// each other's results; the caller must order them.
#include <algorithm>
#include <cstdio>
#include <mutex>

#include "../../include/moestream.h"
#include "host_wait.h"
#include "kernels.h"

using namespace ms;

namespace {

constexpr int MAX_T = MS_STATIC_MAX_TOKENS;
constexpr int MAX_P = MS_STATIC_MAX_PAIRS;
constexpr int MAX_D = 4096;                       // d_model and d_ff
constexpr int MAX_SLOTS = MS_STATIC_MAX_SLOTS;
constexpr int MAX_DEVICES = 64;

constexpr size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Carving of the static scratch array (byte offsets).
constexpr size_t OFF_CTR = 0;                                              // TableCtr (status)
constexpr size_t OFF_CNT = align256(OFF_CTR + sizeof(TableCtr));           // unsigned [MAX_D/16]
constexpr size_t OFF_NGROUPS = align256(OFF_CNT + 4 * (MAX_D / 16));       // int
constexpr size_t ZERO_BYTES = OFF_NGROUPS + 256;                           // cleared every call
constexpr size_t OFF_GKEY = ZERO_BYTES;
constexpr size_t OFF_GSLOT = align256(OFF_GKEY + 4 * MAX_P);
constexpr size_t OFF_GSTART = align256(OFF_GSLOT + 4 * MAX_P);
constexpr size_t OFF_GCOUNT = align256(OFF_GSTART + 4 * MAX_P);
constexpr size_t OFF_GPAIRS = align256(OFF_GCOUNT + 4 * MAX_P);
constexpr size_t OFF_KEYS = align256(OFF_GPAIRS + 4 * MAX_P);
constexpr size_t OFF_MAP = align256(OFF_KEYS + 4 * MAX_P);                 // int [MAX_SLOTS+1]
constexpr size_t OFF_XFRAG = align256(OFF_MAP + 4 * (MAX_SLOTS + 1));      // half [MAX_T*MAX_D]
constexpr size_t OFF_XSUM = align256(OFF_XFRAG + 2 * MAX_T * MAX_D);       // float [MAX_T*MAX_D/64*2]
constexpr size_t OFF_HFRAG = align256(OFF_XSUM + 4 * MAX_T * (MAX_D / 64) * 2);  // half [MAX_P*MAX_D]
constexpr size_t OFF_HPART = align256(OFF_HFRAG + 2 * MAX_P * MAX_D);      // float [MAX_P*MAX_D/16*2]
constexpr size_t OFF_YPART = align256(OFF_HPART + 4 * MAX_P * (MAX_D / 16) * 2);  // float [MAX_P*MAX_D]
constexpr size_t SCRATCH_BYTES = align256(OFF_YPART + 4 * MAX_P * MAX_D);

// The scratch itself. In host code `g_static_scratch` names a host-side
// stand-in, not device memory: its device address is obtained with
// cudaGetSymbolAddress, per device, below.
static __device__ __align__(256) unsigned char g_static_scratch[SCRATCH_BYTES];

std::mutex g_mu;
void* g_dev_ptr[MAX_DEVICES] = {};

int sfail(int code, const char* msg) {
  set_error_message(msg);                      // read back with ms_last_error
  return code;
}

// Device address of the scratch on the current device, looked up on the
// first call made on that device.
int scratch_ptr(unsigned char** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return sfail(MS_E_CUDA, "cudaGetDevice failed");
  if (dev < 0 || dev >= MAX_DEVICES) return sfail(MS_E_INVALID, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_dev_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || !p) {
      char buf[256];
      snprintf(buf, sizeof(buf), "cudaGetSymbolAddress of the static scratch failed: %s",
               cudaGetErrorString(e));
      return sfail(MS_E_CUDA, buf);
    }
    g_dev_ptr[dev] = p;
  }
  *out = static_cast<unsigned char*>(g_dev_ptr[dev]);
  return MS_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int ms_expert_mlp_static(const ms_geom* geom, const void* arena, int n_slots,
                                    const int32_t* slots, const float* scores, const void* x,
                                    int T, int k, void* y, void* stream) {
  if (!geom || !arena || !slots || !scores || !x || !y)
    return sfail(MS_E_INVALID, "ms_expert_mlp_static: NULL argument");
  const ms_geom& g = *geom;
  {
    // the pool path's geometry checks: every component the kernels read
    // (offset plus the size its shape gives) inside the blob
    char msg[256], full[320];
    if (validate_geom(geom, msg, sizeof(msg)) != MS_OK) {
      snprintf(full, sizeof(full), "ms_expert_mlp_static: %s", msg);
      return sfail(MS_E_INVALID, full);
    }
  }
  if (g.d_model > MAX_D || g.d_ff > MAX_D)
    return sfail(MS_E_INVALID, "ms_expert_mlp_static: d_model and d_ff must be <= 4096");
  if (!expert_shape_ok(g.model, g.d_model, g.d_ff))
    return sfail(MS_E_INVALID,
                 "ms_expert_mlp_static: shape not handled by the decode kernels (gpt-oss: d_model "
                 "and d_ff <= 3072)");
  if (k != g.top_k) return sfail(MS_E_INVALID, "ms_expert_mlp_static: k must equal top_k");
  if (T <= 0 || T > MAX_T)
    return sfail(MS_E_INVALID, "ms_expert_mlp_static: T must be in [1, MS_STATIC_MAX_TOKENS]");
  if ((long long)T * k > MAX_P)
    return sfail(MS_E_INVALID, "ms_expert_mlp_static: T*k exceeds MS_STATIC_MAX_PAIRS");
  if (n_slots <= 0 || n_slots > MAX_SLOTS)
    return sfail(MS_E_INVALID, "ms_expert_mlp_static: n_slots must be in [1, MS_STATIC_MAX_SLOTS]");
  if (!aligned16(x) || !aligned16(y) || !aligned16(arena))
    return sfail(MS_E_INVALID, "ms_expert_mlp_static: x, y and arena must be 16-byte aligned");

  unsigned char* base = nullptr;
  int rc = scratch_ptr(&base);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // status, arrival counters and the group count must start at zero
  if (cudaMemsetAsync(base, 0, ZERO_BYTES, s) != cudaSuccess)
    return sfail(MS_E_CUDA, "ms_expert_mlp_static: cudaMemsetAsync failed");

  Geo geo{};
  geo.model = g.model;
  geo.d_model = g.d_model;
  geo.d_ff = g.d_ff;
  geo.n_experts = g.n_experts;
  geo.top_k = g.top_k;
  geo.group_size = g.group_size;
  geo.norm_topk = g.norm_topk_prob;
  geo.proj_bias = g.proj_bias;
  geo.blob = g.blob_bytes;
  for (int a = 0; a < 3; ++a)
    for (int b = 0; b < 4; ++b) geo.off[a][b] = g.comp_offset[a][b];

  Groups grp{};
  grp.n_groups = reinterpret_cast<int*>(base + OFF_NGROUPS);
  grp.grp_key = reinterpret_cast<int*>(base + OFF_GKEY);
  grp.grp_slot = reinterpret_cast<int*>(base + OFF_GSLOT);
  grp.grp_start = reinterpret_cast<int*>(base + OFF_GSTART);
  grp.grp_count = reinterpret_cast<int*>(base + OFF_GCOUNT);
  grp.grp_pairs = reinterpret_cast<int*>(base + OFF_GPAIRS);
  grp.map = reinterpret_cast<int*>(base + OFF_MAP);
  TableCtr* ctr = reinterpret_cast<TableCtr*>(base + OFF_CTR);

  MlpPrepArgs pa{};
  pa.x = static_cast<const uint16_t*>(x);
  pa.T = T;
  pa.k = k;
  pa.d_model = g.d_model;
  pa.n_slots = n_slots;
  pa.slots = slots;
  pa.keys = reinterpret_cast<int*>(base + OFF_KEYS);
  pa.ctr = ctr;
  pa.xfrag = reinterpret_cast<__half*>(base + OFF_XFRAG);
  pa.xsum = reinterpret_cast<float*>(base + OFF_XSUM);
  pa.grp = grp;
  if (launch_mlp_prep(pa, s) != cudaSuccess)
    return sfail(MS_E_CUDA, "ms_expert_mlp_static: prep launch failed");

  ExpArgs e{};
  e.geo = geo;
  e.arena = static_cast<const uint8_t*>(arena);
  e.grp = grp;
  e.T = T;
  e.xfrag = pa.xfrag;
  e.xsum = pa.xsum;
  e.hfrag = reinterpret_cast<__half*>(base + OFF_HFRAG);
  e.hpart = reinterpret_cast<float*>(base + OFF_HPART);
  e.ypart = reinterpret_cast<float*>(base + OFF_YPART);
  e.scores = scores;
  e.cnt = reinterpret_cast<unsigned*>(base + OFF_CNT);
  e.y = static_cast<uint16_t*>(y);
  e.status = &ctr->status;
  if (launch_expert(e, std::min(T * k, n_slots), s) != cudaSuccess)
    return sfail(MS_E_CUDA, "ms_expert_mlp_static: expert kernel launch failed");
  return MS_OK;
}

// Device status of the most recent ms_expert_mlp_static call on the current
// device: an out-of-range slot (its rows come back as zeros) or a bounded
// wait that ran out is recorded in the status word of the static array; this
// reads it after `stream` has finished and clears it. Allocates nothing.
extern "C" int ms_expert_mlp_static_status(void* stream) {
  unsigned char* base = nullptr;
  int rc = scratch_ptr(&base);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = 0;
  TableCtr* ctr = reinterpret_cast<TableCtr*>(base + OFF_CTR);
  if (cudaMemcpyAsync(&st, &ctr->status, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return sfail(MS_E_CUDA, "ms_expert_mlp_static_status: reading the status failed");
  const cudaError_t we = stream_wait_bounded(s);
  if (we == cudaErrorTimeout)
    return sfail(MS_E_TIMEOUT, "ms_expert_mlp_static_status: the stream did not finish within "
                               "the host wait limit (MS_HOST_WAIT_S)");
  if (we != cudaSuccess)
    return sfail(MS_E_CUDA, "ms_expert_mlp_static_status: reading the status failed");
  if (cudaMemsetAsync(&ctr->status, 0, sizeof(int), s) != cudaSuccess ||
      stream_wait_bounded(s) != cudaSuccess)
    return sfail(MS_E_CUDA, "ms_expert_mlp_static_status: clearing the status failed");
  if (st == MS_E_INVALID)
    return sfail(MS_E_INVALID, "ms_expert_mlp_static: a slot index was outside [0, n_slots); "
                               "its rows were returned as zeros");
  if (st == MS_E_TIMEOUT)
    return sfail(MS_E_TIMEOUT, "ms_expert_mlp_static: a bounded wait for the weight copies ran out");
  if (st == MS_E_RANGE)
    return sfail(MS_E_RANGE, "ms_expert_mlp_static: an activation beyond the fp16 range "
                             "(|v| > 65504) reached the expert kernels; the output is not valid");
  if (st) return sfail(st, "ms_expert_mlp_static: device-side error");
  return MS_OK;
}
