// Host side of libmoestream: the C ABI declared in include/moestream.h.
// Owns the slot arena, the device slot table, the mapped store and every
// scratch buffer; launches the kernels of route.cu and expert.cu.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

#include "../../include/moestream.h"
#include "host_wait.h"
#include "kernels.h"
#include "nccl_rt.h"

using namespace ms;

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

#define CK(call)                                                                       \
  do {                                                                                 \
    cudaError_t e_ = (call);                                                           \
    if (e_ != cudaSuccess)                                                             \
      return fail(MS_E_CUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                  __FILE__, __LINE__);                                                 \
  } while (0)

// A host wait on the device (stream_wait_bounded / event_wait_bounded):
// MS_E_TIMEOUT when it ran past the host limit, MS_E_CUDA for a CUDA error.
#define HWAIT(call)                                                                    \
  do {                                                                                 \
    cudaError_t e_ = (call);                                                           \
    if (e_ == cudaErrorTimeout)                                                        \
      return fail(MS_E_TIMEOUT, "%s: the device did not finish within %.0f s "         \
                  "(MS_HOST_WAIT_S)", #call, host_wait_limit_s());                     \
    if (e_ != cudaSuccess)                                                             \
      return fail(MS_E_CUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                  __FILE__, __LINE__);                                                 \
  } while (0)

template <typename T>
int dalloc(T** p, size_t count) {
  *p = nullptr;
  if (count == 0) count = 1;
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T));
  if (e != cudaSuccess)
    return fail(MS_E_NOMEM, "cudaMalloc(%zu bytes): %s", count * sizeof(T), cudaGetErrorString(e));
  return MS_OK;
}

}  // namespace

namespace ms {
void set_error_message(const char* msg) { g_err = msg; }

static int __attribute__((format(printf, 3, 4))) geom_bad(char* msg, size_t n, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(msg, n, fmt, ap);
  va_end(ap);
  return MS_E_INVALID;
}

int validate_geom(const ms_geom* g, char* msg, size_t n) {
#define bad(...) geom_bad(msg, n, __VA_ARGS__)
  if (!g) return bad("geom is NULL");
  if (g->model != MS_MODEL_QWEN3 && g->model != MS_MODEL_GPTOSS) return bad("unknown model %d", g->model);
  if (g->bits != 4 || g->group_size != 64)
    return bad("only 4-bit codes in groups of 64 are supported (got %d bits, group %d)", g->bits,
               g->group_size);
  if (g->d_model <= 0 || g->d_model % 64 || g->d_ff <= 0 || g->d_ff % 64)
    return bad("d_model and d_ff must be positive multiples of 64");
  if (g->d_ff > 4096 || g->d_model > 16384) return bad("d_ff must be <= 4096 and d_model <= 16384");
  if (g->n_experts <= 0 || g->n_experts > 256) return bad("n_experts must be in [1, 256]");
  if (g->top_k <= 0 || g->top_k > 32 || g->top_k > g->n_experts)
    return bad("top_k must be in [1, min(32, n_experts)]");
  if (g->n_layers <= 0) return bad("n_layers must be positive");
  if (g->blob_bytes <= 0 || g->blob_bytes % 16384) return bad("blob_bytes must be a positive multiple of 16384");
  if (g->proj_bias != 0 && g->proj_bias != 1) return bad("proj_bias must be 0 or 1");
  // every component the kernels read lies inside the blob: its offset plus
  // the size the shapes give it (weight U32 [out, in/8], scales and biases
  // BF16 [out, in/64], the projection bias BF16 [out] when proj_bias is set)
  for (int pr = 0; pr < 3; ++pr) {
    const int n_out = pr == 2 ? g->d_model : g->d_ff;
    const int n_in = pr == 2 ? g->d_ff : g->d_model;
    const long long sz[4] = {(long long)n_out * n_in / 2, (long long)n_out * (n_in / 64) * 2,
                             (long long)n_out * (n_in / 64) * 2, (long long)n_out * 2};
    for (int pt = 0; pt < 4; ++pt) {
      const long long off = g->comp_offset[pr][pt];
      if (pt == 3 && !g->proj_bias) continue;
      if (off < 0 || off + sz[pt] > g->blob_bytes)
        return bad("component [%d][%d] at %lld (+%lld) lies outside the blob", pr, pt, off, sz[pt]);
      if (off % 16) return bad("component [%d][%d] is not 16-byte aligned", pr, pt);
    }
  }
#undef bad
  return MS_OK;
}
}  // namespace ms

struct ms_pool {
  int device = 0;
  ms_geom geom{};
  ms_pool_config cfg{};
  Geo geo{};
  long long n_keys = 0;
  int max_pairs = 0;
  int max_groups = 0;
  int sm_count = 148;
  // arena
  uint8_t* arena = nullptr;
  size_t arena_bytes = 0;
  // table
  DevTable tab{};
  std::vector<void*> dev_blocks;
  // store
  uint8_t* store_host = nullptr;
  const uint8_t* store_dev = nullptr;
  size_t store_bytes = 0;
  bool store_owned = false, store_registered = false;
  // routers
  std::vector<const uint16_t*> w_r, b_r;
  // scratch
  float* logits = nullptr;
  unsigned* ticket = nullptr;
  int* inds = nullptr;
  uint16_t* scores = nullptr;
  float* scores_f = nullptr;
  int* pair_slot = nullptr;
  __half* xfrag = nullptr;
  float* xsum = nullptr;
  __half* hfrag = nullptr;
  float* hpart = nullptr;
  float* ypart = nullptr;
  unsigned* cnt = nullptr;
  Groups grp{};
  int* d_slots = nullptr;
  int* d_opstatus = nullptr;
  int* h_pinned = nullptr;   // [MS_MAX_REQ + 1]
  int* mlp_keys = nullptr;     // sanitised slot keys of ms_expert_mlp
  // decode / small batches: the scratch above holds narrow_tokens tokens
  int narrow_tokens = 0;
  // wide batches (prefill): router tiles, grouped tcgen05 GEMM
  bool wide = false;            // scratch and tensor maps ready
  int wide_min_pairs = 0;       // T*k from which ms_moe_block takes this path
  WideArgs wa{};
  long long p_pad = 0;          // rows of xperm / hbuf / ybuf
  uint16_t* xperm = nullptr;
  float* perm_score = nullptr;
  int* inv = nullptr;
  uint16_t* hbuf = nullptr;
  uint16_t* ybuf = nullptr;
  CUtensorMap tm_x{}, tm_h{};
  GemmMaps gm_up{}, gm_dn{};    // code tiles per precision class (gate/up, down)
  // decode expert kernels: gate, up and down weight rows as whole-row tiles
  // (encode_rows_map), when the row widths allow it
  CUtensorMap dec_maps[3] = {};
  bool dec_maps_ok = false;
  int* mlp_cnt = nullptr;       // [n_slots + 1] pairs per slot (wide ms_expert_mlp)
  int* mlp_wkeys = nullptr;     // [max_pairs] sanitised slot keys (wide ms_expert_mlp)
  int* ep_scratch = nullptr;    // [128]: counts and cursors of ms_ep_pack
  bool profile = false;
  std::vector<cudaEvent_t> prof_ev;   // [n_layers][4]
  // prefetch fills of ms_moe_block run on a side stream: forked after the
  // route step, joined before the next call's expert kernels (the only
  // readers of the slots they fill)
  cudaStream_t side = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_pf[2] = {nullptr, nullptr};
  int2* pf_ring = nullptr;      // [2][max_fills]: one half per call, alternating
  int* pf_cnt = nullptr;        // [2] fill counts, [2] error sink of ring fills
  int pf_parity = 0;            // ring half (and event) of the next fork
  bool pf_pending = false;      // ev_pf[pf_slot] not yet joined
  int pf_slot = 0;
  bool pf_captured = false;     // that fork was recorded inside a stream capture
  unsigned long long pf_capture_id = 0;
  // precision classes (ms_pool_set_precision); by default one class, the
  // geometry's 4-bit bf16 blob, served by the tuned uniform kernels
  bool mixed = false;
  bool used = false;            // a slot was filled: the classes are fixed from here on
  ClassTab ctab{};
  long long cls_bytes[MS_MAX_CLASSES] = {};   // bytes a fill of the class copies
  uint8_t* class_of_key = nullptr;            // [n_keys]
  uint8_t* slot_class = nullptr;              // [n_slots]
  std::vector<uint8_t> h_class_of_key;
  // the fused block (ms_moe_block_fused): set for the duration of one call
  const uint16_t* cur_norm_w = nullptr;       // route step normalises its input
  float cur_norm_eps = 0.f;
  const uint16_t* cur_resid = nullptr;        // combines add it to the output
  uint16_t* xnorm = nullptr;                  // [max_tokens, d_model]: normalised input (wide path)
  // expert-parallel group of the C-ABI block (ms_ep_init), or null
  struct EpState* ep = nullptr;
};

// A pool's expert-parallel group: the communicator, the placement, and
// scratch sized by the largest call so far.
struct EpState {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1, e_local = 0, max_rep = 0;
  int32_t* placement = nullptr;   // device [n_experts][1 + 2*max_rep], or null
  int cap_T = 0;                  // local tokens the send side holds
  int32_t* inds = nullptr;        // [cap_T * k]
  uint16_t* scores = nullptr;     // [cap_T * k] bf16
  uint16_t* send_x = nullptr;     // [cap_T * k][d]
  int32_t* send_meta = nullptr;   // [cap_T * k][2]
  int32_t* pair_pos = nullptr;    // [cap_T * k]
  uint16_t* back = nullptr;       // [cap_T * k][d]
  int32_t* counts = nullptr;      // [2][world]: send, receive
  long long cap_recv = 0;         // rows the receive side holds
  uint16_t* recv_x = nullptr;     // [cap_recv][d]
  int32_t* recv_meta = nullptr;   // [cap_recv][2]
  int32_t* recv_slots = nullptr;  // [cap_recv]
  float* recv_scores = nullptr;   // [cap_recv]
  uint16_t* y_recv = nullptr;     // [cap_recv][d]
  int32_t* h_counts = nullptr;    // pinned [2][world]
  // an exchange failed or timed out: operations may be stuck in the
  // communicator, so it is aborted, not destroyed, and not used again
  bool broken = false;
};

static void ep_free_send(EpState* e) {
  for (void* b : {(void*)e->inds, (void*)e->scores, (void*)e->send_x, (void*)e->send_meta,
                  (void*)e->pair_pos, (void*)e->back})
    if (b) cudaFree(b);
  e->inds = nullptr, e->scores = nullptr, e->send_x = nullptr, e->send_meta = nullptr;
  e->pair_pos = nullptr, e->back = nullptr;
  e->cap_T = 0;
}

static void ep_free_recv(EpState* e) {
  for (void* b : {(void*)e->recv_x, (void*)e->recv_meta, (void*)e->recv_slots, (void*)e->recv_scores,
                  (void*)e->y_recv})
    if (b) cudaFree(b);
  e->recv_x = nullptr, e->recv_meta = nullptr, e->recv_slots = nullptr, e->recv_scores = nullptr;
  e->y_recv = nullptr;
  e->cap_recv = 0;
}

static void ep_release(EpState* e) {
  if (!e) return;
  if (e->comm && nccl_rt().ok) {
    if (e->broken) nccl_rt().CommAbort(e->comm);
    else nccl_rt().CommDestroy(e->comm);
  }
  ep_free_send(e);
  ep_free_recv(e);
  if (e->placement) cudaFree(e->placement);
  if (e->counts) cudaFree(e->counts);
  if (e->h_counts) cudaFreeHost(e->h_counts);
  delete e;
}

namespace {

template <typename T>
int palloc(ms_pool* p, T** out, size_t count) {
  int rc = dalloc(out, count);
  if (rc == MS_OK) p->dev_blocks.push_back(*out);
  return rc;
}

int check_geom(const ms_geom* g) {
  char msg[256];
  const int rc = ms::validate_geom(g, msg, sizeof(msg));
  return rc ? fail(rc, "%s", msg) : MS_OK;
}

Geo make_geo(const ms_geom& g) {
  Geo o{};
  o.model = g.model;
  o.d_model = g.d_model;
  o.d_ff = g.d_ff;
  o.n_experts = g.n_experts;
  o.top_k = g.top_k;
  o.group_size = g.group_size;
  o.norm_topk = g.norm_topk_prob;
  o.proj_bias = g.proj_bias;
  o.blob = g.blob_bytes;
  for (int a = 0; a < 3; ++a)
    for (int b = 0; b < 4; ++b) o.off[a][b] = g.comp_offset[a][b];
  return o;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Pair count from which ms_moe_block runs the grouped-GEMM path; calls above
// MS_MLP_MAX_PAIRS pairs always do. MS_WIDE_MIN_PAIRS overrides it.
int wide_threshold() {
  const char* v = getenv("MS_WIDE_MIN_PAIRS");
  if (v && *v) {
    const long t = strtol(v, nullptr, 10);
    if (t > 0) return (int)std::min<long>(t, 1L << 30);
  }
  return 1024;
}

// Scratch and tensor maps of the wide-batch path, when max_tokens reaches it.
int setup_wide(ms_pool* p) {
  const int E = p->geom.n_experts, D = p->geom.d_model, F = p->geom.d_ff;
  p->wide_min_pairs = wide_threshold();
  const long long P = p->max_pairs;
  if (P < std::min<long long>(p->wide_min_pairs, MS_MLP_MAX_PAIRS + 1)) return MS_OK;
  // rows of the GEMM operands: whole 256-row boxes, so no TMA box is taller
  // than its tensor
  p->p_pad = (P + GEMM_TILE_ROWS - 1) / GEMM_TILE_ROWS * GEMM_TILE_ROWS;
  int rc;
  WideArgs& w = p->wa;
  // groups: experts on the routed path, slots (up to n_slots + 1) on the
  // ms_expert_mlp path
  const long long n_keys = std::max<long long>(E, (long long)p->cfg.n_slots + 1);
  w.max_tiles = (int)std::min<long long>(P / GEMM_TILE_ROWS + std::min<long long>(n_keys, P) + 1, 65535);
  if ((rc = palloc(p, &w.cnt_e, 256))) return rc;
  if ((rc = palloc(p, &w.pmask, MS_MAX_DEPTHS * 8))) return rc;
  if ((rc = palloc(p, &w.cursor, std::max<long long>(256, n_keys)))) return rc;
  if ((rc = palloc(p, &p->mlp_cnt, p->cfg.n_slots + 1))) return rc;
  if ((rc = palloc(p, &p->mlp_wkeys, P))) return rc;
  CK(cudaMemset(p->mlp_cnt, 0, sizeof(int) * (p->cfg.n_slots + 1)));
  if ((rc = palloc(p, &w.tiles, w.max_tiles))) return rc;
  if ((rc = palloc(p, &w.n_tiles, 1))) return rc;
  CK(cudaMemset(w.cnt_e, 0, sizeof(int) * 256));
  CK(cudaMemset(w.pmask, 0, sizeof(unsigned) * MS_MAX_DEPTHS * 8));
  CK(cudaMemset(w.cursor, 0, sizeof(int) * 256));
  CK(cudaMemset(w.n_tiles, 0, sizeof(int)));
  if ((rc = palloc(p, &p->xperm, p->p_pad * D))) return rc;
  if ((rc = palloc(p, &p->perm_score, p->p_pad))) return rc;
  if ((rc = palloc(p, &p->inv, P))) return rc;
  if ((rc = palloc(p, &p->hbuf, p->p_pad * F))) return rc;
  if ((rc = palloc(p, &p->ybuf, p->p_pad * D))) return rc;
  const int64_t* o = &p->geom.comp_offset[0][0];
  const int ns = p->cfg.n_slots;
  const long long blob = p->geom.blob_bytes;
  if (encode_act_map(&p->tm_x, p->xperm, D, p->p_pad) || encode_act_map(&p->tm_h, p->hbuf, F, p->p_pad) ||
      encode_codes_map(&p->gm_up.w[0][0], p->arena + o[0 * 4 + 0], D / 2, F, ns, blob, 32, 64) ||
      encode_codes_map(&p->gm_up.w[1][0], p->arena + o[1 * 4 + 0], D / 2, F, ns, blob, 32, 64) ||
      encode_codes_map(&p->gm_dn.w[0][0], p->arena + o[2 * 4 + 0], F / 2, D, ns, blob, 32, 128))
    return fail(MS_E_CUDA, "cuTensorMapEncodeTiled failed for the grouped-GEMM operands");
  p->wide = true;
  return MS_OK;
}

// Code-tile maps of the grouped GEMM for every precision class.
int encode_class_maps(ms_pool* p, const ClassTab& t) {
  const int D = p->geom.d_model, F = p->geom.d_ff, ns = p->cfg.n_slots;
  const long long blob = p->geom.blob_bytes;
  for (int i = 0; i < t.n; ++i) {
    const PrecDev& c = t.c[i];
    const int cb = gemm_tile_row_bytes(c.bits);
    if (encode_codes_map(&p->gm_up.w[0][i], p->arena + c.off[0][P_W], code_row_bytes(D, c.bits), F, ns,
                         blob, cb, 64) ||
        encode_codes_map(&p->gm_up.w[1][i], p->arena + c.off[1][P_W], code_row_bytes(D, c.bits), F, ns,
                         blob, cb, 64) ||
        encode_codes_map(&p->gm_dn.w[0][i], p->arena + c.off[2][P_W], code_row_bytes(F, c.bits), D, ns,
                         blob, cb, 128))
      return fail(MS_E_CUDA, "cuTensorMapEncodeTiled failed for the code tiles of class %d", i);
  }
  return MS_OK;
}

// The geometry's own blob as precision class 0.
void default_classes(ms_pool* p) {
  ClassTab t{};
  t.n = 1;
  t.c[0].bits = 4;
  t.c[0].fmt = SF_BF16;
  for (int a = 0; a < 3; ++a)
    for (int b = 0; b < 4; ++b) t.c[0].off[a][b] = std::max<long long>(0, p->geom.comp_offset[a][b]);
  p->ctab = t;
  p->cls_bytes[0] = p->geom.blob_bytes;
  p->mixed = false;
}

}  // namespace

extern "C" {

int ms_last_error(char* buf, size_t n) {
  if (!buf || n == 0) return MS_E_INVALID;
  snprintf(buf, n, "%s", g_err.c_str());
  return MS_OK;
}

int ms_pool_create(const ms_geom* geom, const ms_pool_config* cfg, int device, ms_pool** out) {
  if (!out) return fail(MS_E_INVALID, "out is NULL");
  *out = nullptr;
  int rc = check_geom(geom);
  if (rc) return rc;
  if (!cfg) return fail(MS_E_INVALID, "cfg is NULL");
  if (cfg->n_slots <= 0 || cfg->n_slots > 262144)
    return fail(MS_E_INVALID, "n_slots must be in [1, 262144]");
  if (cfg->evict < 0 || cfg->evict > 2) return fail(MS_E_INVALID, "unknown evict mode %d", cfg->evict);
  if (cfg->n_depths < 0 || cfg->n_depths > MS_MAX_DEPTHS)
    return fail(MS_E_INVALID, "n_depths must be in [0, %d]", MS_MAX_DEPTHS);
  for (int i = 0; i < cfg->n_depths; ++i)
    if (cfg->depths[i] <= 0) return fail(MS_E_INVALID, "prefetch depths must be positive");
  if (cfg->pf_widen <= 0) return fail(MS_E_INVALID, "pf_widen must be positive");
  if (geom->n_experts * (1 + cfg->n_depths) > 640)
    return fail(MS_E_INVALID, "n_experts * (1 + n_depths) must be <= 640");
  if ((long long)geom->top_k * cfg->pf_widen > geom->n_experts && cfg->n_depths > 0) {
    // engine_v3.py:513 clamps to n_experts
  }
  if (cfg->max_tokens <= 0) return fail(MS_E_INVALID, "max_tokens must be positive");

  int ndev = 0;
  CK(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return fail(MS_E_INVALID, "device %d out of range", device);
  CK(cudaSetDevice(device));

  ms_pool* p = new ms_pool();
  p->device = device;
  p->geom = *geom;
  p->cfg = *cfg;
  p->geo = make_geo(*geom);
  p->n_keys = (long long)geom->n_layers * geom->n_experts;
  p->max_pairs = cfg->max_tokens * geom->top_k;
  p->max_groups = std::min(p->max_pairs, geom->n_experts);
  cudaDeviceGetAttribute(&p->sm_count, cudaDevAttrMultiProcessorCount, device);
  p->w_r.assign(geom->n_layers, nullptr);
  p->b_r.assign(geom->n_layers, nullptr);

  auto bail = [&](int code) {
    ms_pool_destroy(p);
    return code;
  };
  // a failing CUDA call releases what creation had set up so far
#define CKB(call)                                                                  \
  do {                                                                             \
    cudaError_t e_ = (call);                                                       \
    if (e_ != cudaSuccess)                                                         \
      return bail(fail(MS_E_CUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                       __FILE__, __LINE__));                                       \
  } while (0)

  // arena: n_slots blobs, slot s at s*blob (16 KiB aligned: cudaMalloc is 256 B
  // aligned and blob is a multiple of 16 KiB, so every component keeps its
  // store alignment)
  p->arena_bytes = (size_t)cfg->n_slots * (size_t)geom->blob_bytes;
  if ((rc = palloc(p, &p->arena, p->arena_bytes))) return bail(rc);
  if (cudaMemset(p->arena, 0, p->arena_bytes) != cudaSuccess)
    return bail(fail(MS_E_CUDA, "arena memset failed"));

  // slot table
  DevTable& t = p->tab;
  t.n_slots = cfg->n_slots;
  t.n_keys = (int)p->n_keys;
  t.n_experts = geom->n_experts;
  t.evict = cfg->evict;
  t.window = 24 * std::max(1, cfg->n_depths > 0 ? cfg->depths[0] : 1);
  const int kp = std::min(geom->top_k * cfg->pf_widen, geom->n_experts);
  t.max_fills = geom->n_experts * (1 + cfg->n_depths) + 1;
  if ((rc = palloc(p, &t.key_of, t.n_slots))) return bail(rc);
  if ((rc = palloc(p, &t.slot_of, t.n_keys))) return bail(rc);
  if ((rc = palloc(p, &t.freq, t.n_keys))) return bail(rc);
  if ((rc = palloc(p, &t.born, t.n_keys))) return bail(rc);
  if ((rc = palloc(p, &t.last_use, t.n_keys))) return bail(rc);
  if ((rc = palloc(p, &t.kflags, t.n_keys))) return bail(rc);
  if ((rc = palloc(p, &t.pinned, t.n_slots))) return bail(rc);
  if ((rc = palloc(p, &t.pin_list, t.n_slots))) return bail(rc);
  if ((rc = palloc(p, &t.pend_list, t.n_slots))) return bail(rc);
  if ((rc = palloc(p, &t.fills, t.max_fills))) return bail(rc);
  if ((rc = palloc(p, &t.ctr, 1))) return bail(rc);
  if ((rc = palloc(p, &p->xnorm, (size_t)cfg->max_tokens * geom->d_model))) return bail(rc);
  if ((rc = palloc(p, &p->class_of_key, t.n_keys))) return bail(rc);
  if ((rc = palloc(p, &p->slot_class, t.n_slots))) return bail(rc);
  CKB(cudaMemset(p->class_of_key, 0, t.n_keys));
  CKB(cudaMemset(p->slot_class, 0, t.n_slots));
  default_classes(p);
  if ((rc = palloc(p, &p->pf_ring, 2 * (size_t)t.max_fills))) return bail(rc);
  if ((rc = palloc(p, &p->pf_cnt, 3))) return bail(rc);
  CKB(cudaMemset(p->pf_cnt, 0, 3 * sizeof(int)));
  CKB(cudaStreamCreateWithFlags(&p->side, cudaStreamNonBlocking));
  CKB(cudaEventCreateWithFlags(&p->ev_fork, cudaEventDisableTiming));
  for (auto& e : p->ev_pf) CKB(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  CKB(cudaMemset(t.key_of, 0xff, sizeof(int) * t.n_slots));
  CKB(cudaMemset(t.slot_of, 0xff, sizeof(int) * t.n_keys));
  CKB(cudaMemset(t.freq, 0, sizeof(int) * t.n_keys));
  CKB(cudaMemset(t.born, 0, sizeof(long long) * t.n_keys));
  CKB(cudaMemset(t.last_use, 0, sizeof(long long) * t.n_keys));
  CKB(cudaMemset(t.kflags, 0, t.n_keys));
  CKB(cudaMemset(t.pinned, 0, t.n_slots));
  TableCtr c0{};
  c0.n_free = t.n_slots;
  CKB(cudaMemcpy(t.ctr, &c0, sizeof(c0), cudaMemcpyHostToDevice));

  // scratch: routing results for up to max_tokens; the decode-path
  // intermediates for up to narrow_tokens (MS_MLP_MAX_PAIRS pairs)
  const long long P = p->max_pairs;
  const int E = geom->n_experts, D = geom->d_model, F = geom->d_ff;
  p->narrow_tokens = std::min(cfg->max_tokens, MS_MLP_MAX_PAIRS / geom->top_k);
  const long long Tn = p->narrow_tokens, Pn = Tn * geom->top_k;
  if ((rc = palloc(p, &p->logits, Tn * E * (1 + cfg->n_depths)))) return bail(rc);
  if ((rc = palloc(p, &p->ticket, 1))) return bail(rc);
  CKB(cudaMemset(p->ticket, 0, sizeof(unsigned)));
  if ((rc = palloc(p, &p->inds, P))) return bail(rc);
  if ((rc = palloc(p, &p->scores, P))) return bail(rc);
  if ((rc = palloc(p, &p->scores_f, P))) return bail(rc);
  if ((rc = palloc(p, &p->pair_slot, P))) return bail(rc);
  if ((rc = palloc(p, &p->xfrag, Tn * D))) return bail(rc);
  if ((rc = palloc(p, &p->xsum, Tn * (D / 64) * 2))) return bail(rc);
  if ((rc = palloc(p, &p->hfrag, Pn * F))) return bail(rc);
  if ((rc = palloc(p, &p->hpart, Pn * (F / 16) * 2))) return bail(rc);
  if ((rc = palloc(p, &p->ypart, Pn * D))) return bail(rc);
  if ((rc = palloc(p, &p->cnt, D / 16))) return bail(rc);
  CKB(cudaMemset(p->cnt, 0, sizeof(unsigned) * (D / 16)));
  const long long key_range = std::max<long long>(E, cfg->n_slots + 1);
  if ((rc = palloc(p, &p->mlp_keys, std::min<long long>(P, MS_MLP_MAX_PAIRS)))) return bail(rc);
  if ((rc = palloc(p, &p->grp.n_groups, 1))) return bail(rc);
  if ((rc = palloc(p, &p->grp.grp_key, std::max<long long>(P, E)))) return bail(rc);
  if ((rc = palloc(p, &p->grp.grp_slot, std::max<long long>(P, E)))) return bail(rc);
  if ((rc = palloc(p, &p->grp.grp_start, std::max<long long>(P, E)))) return bail(rc);
  if ((rc = palloc(p, &p->grp.grp_count, std::max<long long>(P, E)))) return bail(rc);
  if ((rc = palloc(p, &p->grp.grp_pairs, P))) return bail(rc);
  if ((rc = palloc(p, &p->grp.map, key_range))) return bail(rc);
  CKB(cudaMemset(p->grp.n_groups, 0, sizeof(int)));
  if ((rc = palloc(p, &p->ep_scratch, 128))) return bail(rc);
  if ((rc = palloc(p, &p->d_slots, MS_MAX_REQ))) return bail(rc);
  if ((rc = palloc(p, &p->d_opstatus, 1))) return bail(rc);
  if (cudaMallocHost(reinterpret_cast<void**>(&p->h_pinned), sizeof(int) * (MS_MAX_REQ + 1)) !=
      cudaSuccess)
    return bail(fail(MS_E_NOMEM, "cudaMallocHost failed"));
  (void)kp;
  {
    const int64_t* o = &p->geom.comp_offset[0][0];
    const int dr = expert_down_rows(geom->model, D, F);
    p->dec_maps_ok =
        encode_rows_map(&p->dec_maps[0], p->arena + o[0], D / 2, F, cfg->n_slots, geom->blob_bytes, 16) == 0 &&
        encode_rows_map(&p->dec_maps[1], p->arena + o[4], D / 2, F, cfg->n_slots, geom->blob_bytes, 16) == 0 &&
        encode_rows_map(&p->dec_maps[2], p->arena + o[8], F / 2, D, cfg->n_slots, geom->blob_bytes, dr) == 0;
  }
  // the fill and route kernels run beside the expert kernels (the fills on
  // the side stream): keep every SM on its largest shared-memory split
  CKB(route_prefer_shared());
  if ((rc = setup_wide(p))) return bail(rc);
  CKB(cudaDeviceSynchronize());
#undef CKB
  *out = p;
  return MS_OK;
}

int ms_pool_destroy(ms_pool* p) {
  if (!p) return MS_OK;
  cudaSetDevice(p->device);
  cudaDeviceSynchronize();
  ep_release(p->ep);
  for (void* b : p->dev_blocks) cudaFree(b);
  for (cudaEvent_t e : p->prof_ev) cudaEventDestroy(e);
  if (p->ev_fork) cudaEventDestroy(p->ev_fork);
  for (cudaEvent_t e : p->ev_pf)
    if (e) cudaEventDestroy(e);
  if (p->side) cudaStreamDestroy(p->side);
  if (p->h_pinned) cudaFreeHost(p->h_pinned);
  if (p->store_owned && p->store_host) cudaFreeHost(p->store_host);
  if (p->store_registered && p->store_host) cudaHostUnregister(p->store_host);
  delete p;
  return MS_OK;
}

int ms_store_register(ms_pool* p, void* host, size_t bytes) {
  if (!p || !host) return fail(MS_E_INVALID, "NULL argument");
  const size_t need = (size_t)p->n_keys * (size_t)p->geom.blob_bytes;
  if (bytes < (size_t)p->geom.blob_bytes)
    return fail(MS_E_INVALID, "store of %zu bytes is smaller than one blob", bytes);
  (void)need;
  CK(cudaSetDevice(p->device));
  if (p->store_host) return fail(MS_E_STATE, "a store is already attached");
  cudaPointerAttributes attr{};
  void* dptr = nullptr;
  if (cudaPointerGetAttributes(&attr, host) == cudaSuccess && attr.type == cudaMemoryTypeHost &&
      attr.devicePointer) {
    dptr = attr.devicePointer;
  } else {
    cudaGetLastError();
    CK(cudaHostRegister(host, bytes, cudaHostRegisterMapped | cudaHostRegisterPortable));
    CK(cudaHostGetDevicePointer(&dptr, host, 0));
    p->store_registered = true;
  }
  p->store_host = static_cast<uint8_t*>(host);
  p->store_dev = static_cast<const uint8_t*>(dptr);
  p->store_bytes = bytes;
  return MS_OK;
}

int ms_store_alloc(ms_pool* p, size_t bytes, void** host_out) {
  if (!p || !host_out) return fail(MS_E_INVALID, "NULL argument");
  if (p->store_host) return fail(MS_E_STATE, "a store is already attached");
  CK(cudaSetDevice(p->device));
  void* h = nullptr;
  cudaError_t e = cudaHostAlloc(&h, bytes, cudaHostAllocMapped | cudaHostAllocPortable);
  if (e != cudaSuccess) return fail(MS_E_NOMEM, "cudaHostAlloc(%zu): %s", bytes, cudaGetErrorString(e));
  void* d = nullptr;
  CK(cudaHostGetDevicePointer(&d, h, 0));
  p->store_host = static_cast<uint8_t*>(h);
  p->store_dev = static_cast<const uint8_t*>(d);
  p->store_bytes = bytes;
  p->store_owned = true;
  *host_out = h;
  return MS_OK;
}

int ms_set_router(ms_pool* p, int layer, const void* w_r, const void* b_r) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  if (layer < 0 || layer >= p->geom.n_layers) return fail(MS_E_INVALID, "layer %d out of range", layer);
  if (w_r && !aligned16(w_r)) return fail(MS_E_INVALID, "router weights must be 16-byte aligned");
  p->w_r[layer] = static_cast<const uint16_t*>(w_r);
  p->b_r[layer] = static_cast<const uint16_t*>(b_r);
  return MS_OK;
}

// Make stream s wait for the pending side-stream prefetch fills. Inside a
// capture the wait is a graph edge; fills forked before the capture began
// are waited for on the host instead (a capture cannot depend on them).
static int join_side(ms_pool* p, cudaStream_t s) {
  if (!p->pf_pending) return MS_OK;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  unsigned long long id = 0;
  CK(cudaStreamGetCaptureInfo(s, &cs, &id));
  const bool cap = cs == cudaStreamCaptureStatusActive;
  if (cap == p->pf_captured && (!cap || id == p->pf_capture_id)) {
    CK(cudaStreamWaitEvent(s, p->ev_pf[p->pf_slot], 0));
  } else if (!p->pf_captured) {
    HWAIT(event_wait_bounded(p->ev_pf[p->pf_slot]));
  } else {
    // a capture that ended without joining its fork cannot be waited for
    // from here; report it once and forget the fork
    p->pf_pending = false;
    return fail(MS_E_STATE,
                "prefetch fills forked inside a stream capture were not joined into it "
                "(call ms_pool_join on the capturing stream before ending the capture)");
  }
  p->pf_pending = false;
  return MS_OK;
}

int ms_pool_join(ms_pool* p, void* stream) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  CK(cudaSetDevice(p->device));
  return join_side(p, static_cast<cudaStream_t>(stream));
}

// CTAs of a fill kernel. The store is read over PCIe (~50 GB/s, a few µs
// of latency): 32 CTAs x 16 KiB in flight cover that bandwidth-delay
// product several times over, and more CTAs only crowd the memory pipelines
// of the SMs that the kernels running beside a side-stream fill also use
// (296 CTAs cost the decode stack ~8 % of its throughput).
constexpr int FILL_CTAS = 32;

static FillArgs fill_args(ms_pool* p) {
  p->used = true;                       // fills may run from here on
  FillArgs f{};
  f.store = p->store_dev;
  f.arena = p->arena;
  f.blob = p->geom.blob_bytes;
  f.store_keys = (long long)(p->store_bytes / (size_t)p->geom.blob_bytes);
  f.fills = p->tab.fills;
  f.max_fills = p->tab.max_fills;
  f.ctr = p->tab.ctr;
  f.slot_class = p->slot_class;
  if (p->mixed) {
    f.class_of_key = p->class_of_key;
    for (int i = 0; i < p->ctab.n; ++i) f.cls_chunks[i] = (int)((p->cls_bytes[i] + 16383) / 16384);
  }
  return f;
}

static int pool_op(ms_pool* p, int op, int layer, const int32_t* experts, int n, cudaStream_t s) {
  if (layer < 0 || layer >= p->geom.n_layers) return fail(MS_E_INVALID, "layer %d out of range", layer);
  if (n < 0 || n > MS_MAX_REQ) return fail(MS_E_INVALID, "n=%d: at most %d experts per call", n, MS_MAX_REQ);
  if (n > 0 && !experts) return fail(MS_E_INVALID, "experts is NULL");
  if (!p->store_dev) return fail(MS_E_STATE, "no store attached (ms_store_register / ms_store_alloc)");
  PoolReq r{};
  r.op = op;
  r.layer = layer;
  r.n = n;
  for (int i = 0; i < n; ++i) {
    if (experts[i] < 0 || experts[i] >= p->geom.n_experts)
      return fail(MS_E_INVALID, "expert %d out of range", experts[i]);
    r.experts[i] = experts[i];
  }
  CK(cudaSetDevice(p->device));
  if (int rc = join_side(p, s)) return rc;
  CK(launch_pool_op(p->tab, r, p->d_slots, p->d_opstatus, s));
  CK(launch_fill(fill_args(p), FILL_CTAS, s));
  return MS_OK;
}

int ms_pool_prefetch(ms_pool* p, int layer, const int32_t* experts, int n, void* stream) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  return pool_op(p, 0, layer, experts, n, static_cast<cudaStream_t>(stream));
}

int ms_pool_acquire(ms_pool* p, int layer, const int32_t* experts, int n, int32_t* slots_out,
                    void* stream) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  if (n > 0 && !slots_out) return fail(MS_E_INVALID, "slots_out is NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = pool_op(p, 1, layer, experts, n, s);
  if (rc) return rc;
  if (n > 0) CK(cudaMemcpyAsync(p->h_pinned, p->d_slots, sizeof(int) * n, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(p->h_pinned + MS_MAX_REQ, p->d_opstatus, sizeof(int), cudaMemcpyDeviceToHost, s));
  HWAIT(stream_wait_bounded(s));
  if (p->h_pinned[MS_MAX_REQ] == MS_E_EXHAUSTED)
    return fail(MS_E_EXHAUSTED, "pool exhausted: every slot pinned or pending");
  for (int i = 0; i < n; ++i) slots_out[i] = p->h_pinned[i];
  return MS_OK;
}

int ms_pool_read(ms_pool* p, int slot, int layer, int expert, void* stream) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  if (slot < 0 || slot >= p->cfg.n_slots) return fail(MS_E_INVALID, "slot %d out of range", slot);
  if (layer < 0 || layer >= p->geom.n_layers || expert < 0 || expert >= p->geom.n_experts)
    return fail(MS_E_INVALID, "(layer %d, expert %d) out of range", layer, expert);
  if (!p->store_host) return fail(MS_E_STATE, "no store attached");
  const size_t blob = (size_t)p->geom.blob_bytes;
  const size_t off = ((size_t)layer * p->geom.n_experts + expert) * blob;
  if (off + blob > p->store_bytes)
    return fail(MS_E_IO, "short read: blob (%d, %d) lies past the end of the store", layer, expert);
  CK(cudaSetDevice(p->device));
  if (int rc = join_side(p, static_cast<cudaStream_t>(stream))) return rc;
  p->used = true;
  const int cls = p->mixed ? p->h_class_of_key[(size_t)layer * p->geom.n_experts + expert] : 0;
  const size_t bytes = p->mixed ? (size_t)p->cls_bytes[cls] : blob;
  CK(cudaMemcpyAsync(p->arena + (size_t)slot * blob, p->store_host + off, bytes,
                     cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream)));
  CK(cudaMemsetAsync(p->slot_class + slot, cls, 1, static_cast<cudaStream_t>(stream)));
  return MS_OK;
}

int ms_pool_stats(ms_pool* p, ms_stats* out) {
  if (!p || !out) return fail(MS_E_INVALID, "NULL argument");
  CK(cudaSetDevice(p->device));
  CK(cudaDeviceSynchronize());
  TableCtr c{};
  CK(cudaMemcpy(&c, p->tab.ctr, sizeof(c), cudaMemcpyDeviceToHost));
  out->prefetch = c.st[ST_PREFETCH];
  out->cache = c.st[ST_CACHE];
  out->miss = c.st[ST_MISS];
  out->total = out->prefetch + out->cache + out->miss;
  out->bail = c.st[ST_BAIL];
  out->issued = c.st[ST_ISSUED];
  out->reads = c.st[ST_READS];
  out->exposed = c.st[ST_EXPOSED];
  out->bytes_read = c.st[ST_READS] * p->geom.blob_bytes;
  out->bytes_exposed = c.st[ST_EXPOSED] * p->geom.blob_bytes;
  return MS_OK;
}

int ms_pool_slot_table(ms_pool* p, int32_t* out) {
  if (!p || !out) return fail(MS_E_INVALID, "NULL argument");
  CK(cudaSetDevice(p->device));
  CK(cudaDeviceSynchronize());
  CK(cudaMemcpy(out, p->tab.key_of, sizeof(int) * p->cfg.n_slots, cudaMemcpyDeviceToHost));
  return MS_OK;
}

int ms_pool_component_ptr(ms_pool* p, int proj, int part, void** out) {
  if (!p || !out) return fail(MS_E_INVALID, "NULL argument");
  if (proj < 0 || proj > 2 || part < 0 || part > 3) return fail(MS_E_INVALID, "bad component");
  const long long off = p->geom.comp_offset[proj][part];
  if (off < 0 || (part == 3 && !p->geom.proj_bias)) return fail(MS_E_INVALID, "component absent");
  *out = p->arena + off;
  return MS_OK;
}

int ms_pool_arena(ms_pool* p, void** base, size_t* bytes) {
  if (!p || !base || !bytes) return fail(MS_E_INVALID, "NULL argument");
  *base = p->arena;
  *bytes = p->arena_bytes;
  return MS_OK;
}

static int route_common(ms_pool* p, int layer, const void* x, int T, cudaStream_t s, bool block,
                        bool wide, int32_t* inds_out, void* scores_out, int32_t* pred_out,
                        int ring = -1) {
  if (layer < 0 || layer >= p->geom.n_layers) return fail(MS_E_INVALID, "layer %d out of range", layer);
  if (T <= 0 || T > p->cfg.max_tokens)
    return fail(MS_E_INVALID, "T=%d outside [1, max_tokens=%d]", T, p->cfg.max_tokens);
  if (!x || !aligned16(x)) return fail(MS_E_INVALID, "x must be a 16-byte aligned device pointer");
  if (!p->w_r[layer]) return fail(MS_E_STATE, "no router set for layer %d", layer);
  RouteArgs a{};
  a.geo = p->geo;
  a.x = static_cast<const uint16_t*>(x);
  a.T = T;
  a.w_r = p->w_r[layer];
  a.b_r = p->b_r[layer];
  a.n_pred = 0;
  for (int i = 0; i < p->cfg.n_depths; ++i) {
    if (!block && (i > 0 || !pred_out)) break;
    const int tgt = layer + p->cfg.depths[i];
    // targets past the last layer are skipped (engine_v3.py:511-512)
    if (tgt >= p->geom.n_layers) continue;
    if (!p->w_r[tgt]) return fail(MS_E_STATE, "no router set for prefetch target layer %d", tgt);
    a.w_p[a.n_pred] = p->w_r[tgt];
    a.b_p[a.n_pred] = p->b_r[tgt];
    a.pred_layer[a.n_pred] = tgt;
    a.n_pred++;
  }
  if (!block && pred_out && a.n_pred == 0)
    return fail(MS_E_INVALID, "layer %d has no prefetch target", layer);
  a.kp = std::min(p->geom.top_k * p->cfg.pf_widen, p->geom.n_experts);
  a.logits = p->logits;
  a.ticket = p->ticket;
  a.inds = inds_out ? inds_out : p->inds;
  a.scores = scores_out ? static_cast<uint16_t*>(scores_out) : p->scores;
  a.scores_f = p->scores_f;
  a.pred_out = pred_out;
  a.xfrag = (block && !wide) ? p->xfrag : nullptr;
  a.xsum = p->xsum;
  a.do_pool = block ? 1 : 0;
  a.tab = p->tab;
  a.layer = layer;
  a.do_groups = block ? 1 : 0;
  a.grp = p->grp;
  a.pair_slot = block ? p->pair_slot : nullptr;
  if (block && !wide && p->cur_norm_w) {
    a.norm_w = p->cur_norm_w;
    a.norm_eps = p->cur_norm_eps;
  }
  if (ring >= 0) {
    a.pf_ring = p->pf_ring + (size_t)ring * p->tab.max_fills;
    a.pf_cnt = p->pf_cnt + ring;
  }
  CK(cudaSetDevice(p->device));
  if (wide) {
    CK(launch_route_wide(a, p->wa, s));
    return MS_OK;
  }
  const int rows = p->geom.n_experts * (1 + a.n_pred);
  int grid = (rows + 7) / 8;
  const int xt = block ? (T * (p->geom.d_model / 64) + 255) / 256 : 0;
  grid = std::max(grid, xt);
  grid = std::min(grid, p->sm_count * 4);
  CK(launch_route_step(a, grid, s));
  return MS_OK;
}

int ms_route(ms_pool* p, int layer, const void* x, int T, int32_t* inds, void* scores,
             int32_t* pred, void* stream) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  if (!inds || !scores) return fail(MS_E_INVALID, "inds/scores are NULL");
  if (pred && p->cfg.n_depths == 0) return fail(MS_E_INVALID, "pred requested but no prefetch depth configured");
  // the router ms_moe_block would use for this batch: the tiled router for
  // wide batches (and whenever the batch exceeds the decode scratch)
  const bool wide = T > p->narrow_tokens ||
                    (p->wide && (long long)T * p->geom.top_k >= p->wide_min_pairs);
  return route_common(p, layer, x, T, static_cast<cudaStream_t>(stream), false, wide, inds, scores,
                      pred);
}

static ExpArgs exp_args(ms_pool* p, const void* x, int T, void* y, const float* scores) {
  (void)x;
  ExpArgs e{};
  e.geo = p->geo;
  e.arena = p->arena;
  e.grp = p->grp;
  e.T = T;
  e.xfrag = p->xfrag;
  e.xsum = p->xsum;
  e.hfrag = p->hfrag;
  e.hpart = p->hpart;
  e.ypart = p->ypart;
  e.scores = scores;
  e.cnt = p->cnt;
  e.y = static_cast<uint16_t*>(y);
  e.status = &p->tab.ctr->status;
  e.slot_class = p->slot_class;
  e.resid = p->cur_resid;
  return e;
}

// The decode expert kernels of the pool: the tuned uniform ones, or the
// per-class ones of a pool with precision classes.
static cudaError_t run_experts(ms_pool* p, const ExpArgs& e, int max_groups, cudaStream_t s) {
  if (p->mixed) return launch_expert_mx(e, p->ctab, max_groups, s);
  return launch_expert(e, max_groups, s, p->dec_maps_ok ? p->dec_maps : nullptr);
}

// Expert MLPs of a routed wide batch: pairs scattered into expert order,
// the two grouped GEMMs, the weighted combine.
// keys: the group key of every pair (expert id after the wide router, slot
// after launch_mlp_wide_prep); the groups and tiles are already laid out.
static int wide_experts(ms_pool* p, const void* x, int T, int k, const int* keys,
                        const float* scores, int* pair_slot, void* y, cudaStream_t s) {
  const int P = T * k;
  ScatterArgs sa{};
  sa.x = static_cast<const uint16_t*>(x);
  sa.T = T;
  sa.k = k;
  sa.d = p->geom.d_model;
  sa.inds = keys;
  sa.scores_f = scores;
  sa.grp = p->grp;
  sa.cursor = p->wa.cursor;
  sa.xperm = p->xperm;
  sa.perm_score = p->perm_score;
  sa.inv = p->inv;
  sa.pair_slot = pair_slot;
  sa.status = &p->tab.ctr->status;
  CK(launch_scatter(sa, std::min((P + 7) / 8, p->sm_count * 8), s));
  GemmArgs g{};
  g.model = p->geo.model;
  g.arena = p->arena;
  g.blob = p->geom.blob_bytes;
  for (int a = 0; a < 3; ++a)
    for (int b = 0; b < 4; ++b) g.off[a][b] = p->geom.comp_offset[a][b];
  g.tiles = p->wa.tiles;
  g.n_tiles = p->wa.n_tiles;
  g.H = p->hbuf;
  g.Y = p->ybuf;
  g.perm_score = p->perm_score;
  g.status = &p->tab.ctr->status;
  const int tiles = (int)std::min<long long>(
      p->wa.max_tiles, P / GEMM_TILE_ROWS + std::min(P, p->geom.n_experts) + 1);
  g.K = p->geom.d_model;
  g.n_out = p->geom.d_ff;
  g.ld_out = p->geom.d_ff;
  g.slot_class = p->slot_class;
  g.C = p->ctab;
  CK(launch_gemm(0, p->tm_x, p->gm_up, g, p->mixed, tiles * (p->geom.d_ff / 64), p->sm_count, s));
  g.K = p->geom.d_ff;
  g.n_out = p->geom.d_model;
  g.ld_out = p->geom.d_model;
  CK(launch_gemm(1, p->tm_h, p->gm_dn, g, p->mixed, tiles * ((p->geom.d_model + 127) / 128),
                 p->sm_count, s));
  CombineArgs c{};
  c.Y = p->ybuf;
  c.inv = p->inv;
  c.y = static_cast<uint16_t*>(y);
  c.T = T;
  c.k = k;
  c.d = p->geom.d_model;
  c.resid = p->cur_resid;
  const long long chunks = (long long)T * (c.d / 8);
  CK(launch_combine(c, (int)std::min<long long>((chunks + 255) / 256, p->sm_count * 8), s));
  return MS_OK;
}

int ms_moe_block(ms_pool* p, int layer, const void* x, int T, void* y, void* stream) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  if (!y || !aligned16(y)) return fail(MS_E_INVALID, "y must be a 16-byte aligned device pointer");
  if (!p->store_dev) return fail(MS_E_STATE, "no store attached (ms_store_register / ms_store_alloc)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaEvent_t* ev = (p->profile && layer >= 0 && layer < p->geom.n_layers)
                        ? &p->prof_ev[(size_t)layer * 4] : nullptr;
  // inside a stream capture an event record must be an external node to be
  // timeable after replay
  unsigned rec_flags = cudaEventRecordDefault;
  if (ev) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    CK(cudaStreamIsCapturing(s, &cs));
    if (cs == cudaStreamCaptureStatusActive) rec_flags = cudaEventRecordExternal;
    CK(cudaEventRecordWithFlags(ev[0], s, rec_flags));
  }
  const int k = p->geom.top_k;
  const bool wide = p->wide && (T * k >= p->wide_min_pairs || T > p->narrow_tokens);
  if (!wide && T > p->narrow_tokens)
    return fail(MS_E_INVALID, "T=%d exceeds the %d tokens of the decode scratch", T, p->narrow_tokens);
  // decode: this call's prefetch fills (slots of later layers) go to the
  // side stream and overlap everything up to the next call's expert kernels
  bool fork = false;
  for (int i = 0; i < p->cfg.n_depths; ++i) fork |= layer + p->cfg.depths[i] < p->geom.n_layers;
  fork = fork && !wide;
  const int q = p->pf_parity;
  int rc = route_common(p, layer, x, T, s, true, wide, nullptr, nullptr, nullptr, fork ? q : -1);
  if (rc) return rc;
  if (ev) CK(cudaEventRecordWithFlags(ev[1], s, rec_flags));
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  unsigned long long cap_id = 0;
  if (fork) {
    CK(cudaStreamGetCaptureInfo(s, &cs, &cap_id));
    CK(cudaEventRecord(p->ev_fork, s));
    CK(cudaStreamWaitEvent(p->side, p->ev_fork, 0));
    FillArgs f = fill_args(p);
    f.ring = p->pf_ring + (size_t)q * p->tab.max_fills;
    f.ring_cnt = p->pf_cnt + q;
    f.ring_err = p->pf_cnt + 2;
    CK(launch_fill(f, FILL_CTAS, p->side));
    CK(cudaEventRecord(p->ev_pf[q], p->side));
  }
  FillArgs fa = fill_args(p);
  fa.acquire_only = fork ? 1 : 0;
  fa.pdl = (fork && !ev) ? 1 : 0;
  // the next layer's call reads the router of layer+1+depth for its
  // speculation before anything else, usually its first touch this step
  if (!wide && p->cfg.n_depths > 0) {
    const int nxt = layer + 1 + p->cfg.depths[0];
    if (nxt < p->geom.n_layers && p->w_r[nxt]) {
      fa.l2_next = p->w_r[nxt];
      fa.l2_next_bytes = (unsigned)((size_t)p->geom.n_experts * p->geom.d_model * 2) & ~15u;
    }
  }
  CK(launch_fill(fa, FILL_CTAS, s));
  // the previous call's prefetch fills must land before any expert kernel
  rc = join_side(p, s);
  // (profiling: the fill interval ends after that join, so the expert
  // interval times the expert kernels alone)
  if (ev && !rc) CK(cudaEventRecordWithFlags(ev[2], s, rec_flags));
  if (fork) {
    p->pf_pending = true;
    p->pf_slot = q;
    p->pf_captured = cs == cudaStreamCaptureStatusActive;
    p->pf_capture_id = cap_id;
    p->pf_parity = q ^ 1;
  }
  if (rc) return rc;
  if (wide) {
    if ((rc = wide_experts(p, x, T, k, p->inds, p->scores_f, p->pair_slot, y, s))) return rc;
  } else {
    const int max_groups = std::min(T * k, p->geom.n_experts);
    ExpArgs e = exp_args(p, x, T, y, p->scores_f);
    // one token: the route step groups the token's k distinct experts one
    // per group, in rank order (its k <= 32 path)
    if (T == 1 && k <= 32 && std::min(k * p->cfg.pf_widen, p->geom.n_experts) <= 32) e.cl_k = k;
    CK(run_experts(p, e, max_groups, s));
  }
  if (ev) CK(cudaEventRecordWithFlags(ev[3], s, rec_flags));
  return MS_OK;
}

// Token rows up to which the route step normalises its own input; larger
// decode batches and the wide path normalise with one kernel first.
constexpr int FUSED_NORM_MAX_T = 8;

int ms_moe_block_fused(ms_pool* p, int layer, const void* h, const void* norm_w, float eps, int T,
                       void* out, void* stream) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  if (!h || !aligned16(h) || !norm_w || !aligned16(norm_w))
    return fail(MS_E_INVALID, "h and norm_w must be 16-byte aligned device pointers");
  if (!(eps > 0.f)) return fail(MS_E_INVALID, "eps must be positive");
  if (T <= 0 || T > p->cfg.max_tokens)
    return fail(MS_E_INVALID, "T=%d outside [1, max_tokens=%d]", T, p->cfg.max_tokens);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int k = p->geom.top_k;
  const bool wide = p->wide && (T * k >= p->wide_min_pairs || T > p->narrow_tokens);
  const void* x = h;
  CK(cudaSetDevice(p->device));
  if (!wide && T <= FUSED_NORM_MAX_T) {
    p->cur_norm_w = static_cast<const uint16_t*>(norm_w);
    p->cur_norm_eps = eps;
  } else {
    CK(launch_rmsnorm(static_cast<const uint16_t*>(h), static_cast<const uint16_t*>(norm_w), eps, T,
                      p->geom.d_model, p->xnorm, s));
    x = p->xnorm;
  }
  p->cur_resid = static_cast<const uint16_t*>(h);
  const int rc = ms_moe_block(p, layer, x, T, out, stream);
  p->cur_norm_w = nullptr;
  p->cur_resid = nullptr;
  return rc;
}

int ms_pool_status(ms_pool* p, void* stream) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CK(cudaSetDevice(p->device));
  if (int rc = join_side(p, s)) return rc;
  HWAIT(stream_wait_bounded(s));
  int st = 0, st_pf = 0;
  CK(cudaMemcpy(&st, &p->tab.ctr->status, sizeof(int), cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(&st_pf, p->pf_cnt + 2, sizeof(int), cudaMemcpyDeviceToHost));
  int zero = 0;
  CK(cudaMemcpy(&p->tab.ctr->status, &zero, sizeof(int), cudaMemcpyHostToDevice));
  CK(cudaMemcpy(p->pf_cnt + 2, &zero, sizeof(int), cudaMemcpyHostToDevice));
  if (!st) st = st_pf;
  if (st == MS_E_EXHAUSTED) return fail(st, "pool exhausted: every slot pinned or pending");
  if (st == MS_E_RANGE)
    return fail(st, "an activation beyond the fp16 range (|v| > 65504) reached the expert "
                    "kernels in an earlier block call; its output is not valid");
  if (st) return fail(st, "device-side error %d in an earlier block call", st);
  return MS_OK;
}

int ms_expert_mlp(ms_pool* p, const int32_t* slots, const float* scores, const void* x, int T,
                  int k, void* y, void* stream) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  if (!slots || !scores || !x || !y) return fail(MS_E_INVALID, "NULL argument");
  if (k <= 0 || k > p->geom.top_k) return fail(MS_E_INVALID, "k=%d outside [1, top_k=%d]", k, p->geom.top_k);
  if (T <= 0) return fail(MS_E_INVALID, "T=%d must be positive", T);
  if (!aligned16(x) || !aligned16(y)) return fail(MS_E_INVALID, "x and y must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CK(cudaSetDevice(p->device));
  if (int rc = join_side(p, s)) return rc;
  // wide batches (and any k other than top_k): slot-keyed grouped GEMM
  const long long P = (long long)T * k;
  const bool wide = p->wide && P <= p->max_pairs &&
                    (k != p->geom.top_k || P >= p->wide_min_pairs || P > MS_MLP_MAX_PAIRS);
  if (wide) {
    MlpWideArgs m{};
    m.slots = slots;
    m.P = (int)P;
    m.n_slots = p->cfg.n_slots;
    m.keys = p->mlp_wkeys;
    m.cnt = p->mlp_cnt;
    m.status = &p->tab.ctr->status;
    m.grp = p->grp;
    m.w = p->wa;
    CK(launch_mlp_wide_prep(m, p->sm_count, s));
    return wide_experts(p, x, T, k, p->mlp_wkeys, scores, nullptr, y, s);
  }
  if (k != p->geom.top_k)
    return fail(MS_E_INVALID, "k=%d != top_k=%d needs the wide path (max_tokens * top_k >= %d pairs)",
                k, p->geom.top_k, p->wide_min_pairs);
  if (T > p->cfg.max_tokens || P > MS_MLP_MAX_PAIRS)
    return fail(MS_E_INVALID, "T=%d outside [1, min(max_tokens, %d/k)]", T, MS_MLP_MAX_PAIRS);
  MlpPrepArgs a{};
  a.x = static_cast<const uint16_t*>(x);
  a.T = T;
  a.k = k;
  a.d_model = p->geom.d_model;
  a.n_slots = p->cfg.n_slots;
  a.slots = slots;
  a.keys = p->mlp_keys;
  a.ctr = p->tab.ctr;
  a.xfrag = p->xfrag;
  a.xsum = p->xsum;
  a.grp = p->grp;
  CK(launch_mlp_prep(a, s));
  CK(run_experts(p, exp_args(p, x, T, y, scores), std::min(T * k, p->cfg.n_slots), s));
  return MS_OK;
}

int ms_ep_pack(ms_pool* p, const void* x, int T, const int32_t* inds, const void* scores, int world,
               int e_local, const int32_t* placement, int max_rep, void* send_x,
               int32_t* send_meta, int32_t* send_counts, int32_t* pair_pos, void* stream) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  if (!x || !inds || !scores || !send_x || !send_meta || !send_counts || !pair_pos)
    return fail(MS_E_INVALID, "NULL argument");
  if (T <= 0) return fail(MS_E_INVALID, "T=%d must be positive", T);
  if (world <= 0 || world > 64) return fail(MS_E_INVALID, "world=%d outside [1, 64]", world);
  if (!placement && (e_local <= 0 || (long long)e_local * world != p->geom.n_experts))
    return fail(MS_E_INVALID, "e_local=%d x world=%d must equal n_experts=%d", e_local, world,
                p->geom.n_experts);
  if (placement && (max_rep <= 0 || max_rep > world))
    return fail(MS_E_INVALID, "max_rep=%d outside [1, world=%d]", max_rep, world);
  if (!aligned16(x) || !aligned16(send_x)) return fail(MS_E_INVALID, "x and send_x must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CK(cudaSetDevice(p->device));
  int* cursor = p->ep_scratch;
  CK(cudaMemsetAsync(send_counts, 0, sizeof(int) * world, s));
  CK(cudaMemsetAsync(cursor, 0, sizeof(int) * world, s));
  EpPackArgs a{};
  a.x = static_cast<const uint16_t*>(x);
  a.T = T;
  a.k = p->geom.top_k;
  a.d = p->geom.d_model;
  a.inds = inds;
  a.scores = static_cast<const uint16_t*>(scores);
  a.world = world;
  a.e_local = e_local;
  a.placement = placement;
  a.max_rep = max_rep;
  a.send_x = static_cast<uint16_t*>(send_x);
  a.send_meta = send_meta;
  a.counts = send_counts;
  a.cursor = cursor;
  a.pair_pos = pair_pos;
  CK(launch_ep_pack(a, p->sm_count, s));
  return MS_OK;
}

int ms_ep_combine(ms_pool* p, const void* back, const int32_t* pair_pos, int T, void* y,
                  void* stream) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  if (!back || !pair_pos || !y) return fail(MS_E_INVALID, "NULL argument");
  if (T <= 0) return fail(MS_E_INVALID, "T=%d must be positive", T);
  if (!aligned16(back) || !aligned16(y)) return fail(MS_E_INVALID, "back and y must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CK(cudaSetDevice(p->device));
  CombineArgs c{};
  c.Y = static_cast<const uint16_t*>(back);
  c.inv = pair_pos;
  c.y = static_cast<uint16_t*>(y);
  c.T = T;
  c.k = p->geom.top_k;
  c.d = p->geom.d_model;
  const long long chunks = (long long)T * (c.d / 8);
  CK(launch_combine(c, (int)std::min<long long>((chunks + 255) / 256, p->sm_count * 8), s));
  return MS_OK;
}

// ------------------------------------------------- expert parallelism, C ABI
#define NCK(call)                                                                      \
  do {                                                                                 \
    const ncclResult_t r_ = (call);                                                    \
    if (r_ != ncclSuccess)                                                             \
      return fail(MS_E_CUDA, "%s failed: %s", #call, nccl_rt().GetErrorString(r_));   \
  } while (0)

int ms_ep_unique_id(uint8_t out[128]) {
  if (!out) return fail(MS_E_INVALID, "NULL argument");
  const NcclRt& rt = nccl_rt();
  if (!rt.ok) return fail(MS_E_CUDA, "NCCL unavailable: %s", rt.why);
  ncclUniqueId id;
  NCK(rt.GetUniqueId(&id));
  static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
  memcpy(out, &id, sizeof(id));
  return MS_OK;
}

int ms_ep_init(ms_pool* p, const uint8_t id[128], int rank, int world, const int32_t* placement,
               int max_rep) {
  if (!p || !id) return fail(MS_E_INVALID, "NULL argument");
  if (p->ep) return fail(MS_E_STATE, "the pool already belongs to an expert-parallel group");
  if (world < 1 || world > 64 || rank < 0 || rank >= world)
    return fail(MS_E_INVALID, "rank=%d / world=%d outside 0 <= rank < world <= 64", rank, world);
  const int E = p->geom.n_experts;
  if (!placement && E % world) return fail(MS_E_INVALID, "%d experts do not shard over %d ranks", E, world);
  if (placement && (max_rep < 1 || max_rep > world))
    return fail(MS_E_INVALID, "max_rep=%d outside [1, world=%d]", max_rep, world);
  if (placement) {
    // every replica's (rank, slot) inside the group and the pool
    for (int e = 0; e < E; ++e) {
      const int32_t* row = placement + (size_t)e * (1 + 2 * max_rep);
      if (row[0] < 1 || row[0] > max_rep)
        return fail(MS_E_INVALID, "placement: expert %d has %d replicas", e, row[0]);
      for (int i = 0; i < row[0]; ++i)
        if (row[1 + 2 * i] < 0 || row[1 + 2 * i] >= world || row[2 + 2 * i] < 0 ||
            row[2 + 2 * i] >= p->cfg.n_slots)
          return fail(MS_E_INVALID, "placement: expert %d replica %d outside the ranks or slots", e, i);
    }
  }
  const NcclRt& rt = nccl_rt();
  if (!rt.ok) return fail(MS_E_CUDA, "NCCL unavailable: %s", rt.why);
  CK(cudaSetDevice(p->device));
  EpState* e = new EpState();
  e->rank = rank;
  e->world = world;
  e->e_local = E / world;
  auto bail = [&](int rc) {
    ep_release(e);
    return rc;
  };
  if (placement) {
    e->max_rep = max_rep;
    const size_t n = (size_t)E * (1 + 2 * max_rep);
    if (int rc = dalloc(&e->placement, n)) return bail(rc);
    if (cudaMemcpy(e->placement, placement, n * sizeof(int32_t), cudaMemcpyHostToDevice) != cudaSuccess)
      return bail(fail(MS_E_CUDA, "placement copy failed"));
  }
  if (int rc = dalloc(&e->counts, 2 * (size_t)world)) return bail(rc);
  if (cudaMallocHost(reinterpret_cast<void**>(&e->h_counts), 2 * world * sizeof(int32_t)) != cudaSuccess)
    return bail(fail(MS_E_NOMEM, "pinned counts"));
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  const ncclResult_t r = rt.CommInitRank(&e->comm, world, uid, rank);
  if (r != ncclSuccess) {
    e->comm = nullptr;
    return bail(fail(MS_E_CUDA, "ncclCommInitRank failed: %s", rt.GetErrorString(r)));
  }
  p->ep = e;
  return MS_OK;
}

int ms_ep_finalize(ms_pool* p) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  if (!p->ep) return MS_OK;
  CK(cudaSetDevice(p->device));
  CK(cudaDeviceSynchronize());
  ep_release(p->ep);
  p->ep = nullptr;
  return MS_OK;
}

// inside ms_ep_moe_block: an NCCL failure also breaks the group
#define NCKB(call)                                                                     \
  do {                                                                                 \
    const ncclResult_t r_ = (call);                                                    \
    if (r_ != ncclSuccess) {                                                           \
      e->broken = true;                                                                \
      return fail(MS_E_CUDA, "%s failed: %s", #call, nccl_rt().GetErrorString(r_));   \
    }                                                                                  \
  } while (0)

int ms_ep_moe_block(ms_pool* p, int layer, const void* x, int T, void* y, void* stream) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  EpState* e = p->ep;
  if (!e) return fail(MS_E_STATE, "no expert-parallel group (ms_ep_init)");
  if (e->broken)
    return fail(MS_E_STATE, "the expert-parallel group failed earlier; ms_ep_finalize it and join a new one");
  if (!x || !y) return fail(MS_E_INVALID, "NULL argument");
  if (T <= 0) return fail(MS_E_INVALID, "T=%d must be positive", T);
  const NcclRt& rt = nccl_rt();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CK(cudaSetDevice(p->device));
  const int k = p->geom.top_k, d = p->geom.d_model, W = e->world;
  const long long P = (long long)T * k;
  // send-side scratch for T local tokens
  if (T > e->cap_T) {
    HWAIT(stream_wait_bounded(s));       // the old buffers may still be in use on s
    ep_free_send(e);
    int rc;
    if ((rc = dalloc(&e->inds, P)) || (rc = dalloc(&e->scores, P)) || (rc = dalloc(&e->send_x, P * d)) ||
        (rc = dalloc(&e->send_meta, 2 * P)) || (rc = dalloc(&e->pair_pos, P)) ||
        (rc = dalloc(&e->back, P * d))) {
      ep_free_send(e);
      return rc;
    }
    e->cap_T = T;
  }
  // 1-2. route and pack (destination-major)
  if (int rc = ms_route(p, layer, x, T, e->inds, e->scores, nullptr, stream)) return rc;
  if (int rc = ms_ep_pack(p, x, T, e->inds, e->scores, W, e->e_local, e->placement,
                          e->placement ? e->max_rep : 0, e->send_x, e->send_meta, e->counts,
                          e->pair_pos, stream))
    return rc;
  // 3. pair counts, then (once the host knows them) the rows and metadata
  int32_t* recv_counts = e->counts + W;
  NCKB(rt.GroupStart());
  for (int r = 0; r < W; ++r) {
    NCKB(rt.Send(e->counts + r, 1, ncclInt32, r, e->comm, s));
    NCKB(rt.Recv(recv_counts + r, 1, ncclInt32, r, e->comm, s));
  }
  NCKB(rt.GroupEnd());
  CK(cudaMemcpyAsync(e->h_counts, e->counts, 2 * W * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  const cudaError_t we = stream_wait_bounded(s);   // a rank that never sends ends here
  if (we != cudaSuccess) e->broken = true;
  HWAIT(we);
  const int32_t* sc = e->h_counts;
  const int32_t* rcn = e->h_counts + W;
  std::vector<long long> soff(W + 1, 0), roff(W + 1, 0);
  for (int r = 0; r < W; ++r) {
    if (sc[r] < 0 || rcn[r] < 0) return fail(MS_E_CUDA, "expert-parallel counts corrupt");
    soff[r + 1] = soff[r] + sc[r];
    roff[r + 1] = roff[r] + rcn[r];
  }
  if (soff[W] != P) return fail(MS_E_CUDA, "ms_ep_pack sent %lld of %lld pairs", soff[W], P);
  const long long n_recv = roff[W];
  if (n_recv > p->cfg.max_tokens)
    return fail(MS_E_INVALID, "%lld rows received, more than the pool's max_tokens=%d", n_recv,
                p->cfg.max_tokens);
  if (n_recv > e->cap_recv) {
    ep_free_recv(e);
    int rc;
    if ((rc = dalloc(&e->recv_x, n_recv * d)) || (rc = dalloc(&e->recv_meta, 2 * n_recv)) ||
        (rc = dalloc(&e->recv_slots, n_recv)) || (rc = dalloc(&e->recv_scores, n_recv)) ||
        (rc = dalloc(&e->y_recv, n_recv * d))) {
      ep_free_recv(e);
      return rc;
    }
    e->cap_recv = n_recv;
  }
  NCKB(rt.GroupStart());
  for (int r = 0; r < W; ++r) {
    if (sc[r]) {
      NCKB(rt.Send(e->send_x + soff[r] * d, (size_t)sc[r] * d * 2, ncclUint8, r, e->comm, s));
      NCKB(rt.Send(e->send_meta + soff[r] * 2, (size_t)sc[r] * 2, ncclInt32, r, e->comm, s));
    }
    if (rcn[r]) {
      NCKB(rt.Recv(e->recv_x + roff[r] * d, (size_t)rcn[r] * d * 2, ncclUint8, r, e->comm, s));
      NCKB(rt.Recv(e->recv_meta + roff[r] * 2, (size_t)rcn[r] * 2, ncclInt32, r, e->comm, s));
    }
  }
  NCKB(rt.GroupEnd());
  // 4. the received rows through this rank's experts, k = 1 (score folded in)
  if (n_recv > 0) {
    CK(cudaMemcpy2DAsync(e->recv_slots, 4, e->recv_meta, 8, 4, n_recv, cudaMemcpyDeviceToDevice, s));
    CK(cudaMemcpy2DAsync(e->recv_scores, 4, e->recv_meta + 1, 8, 4, n_recv, cudaMemcpyDeviceToDevice, s));
    if (int rc = ms_expert_mlp(p, e->recv_slots, e->recv_scores, e->recv_x, (int)n_recv, 1, e->y_recv,
                               stream))
      return rc;
  }
  // 5. the rows back to their senders
  NCKB(rt.GroupStart());
  for (int r = 0; r < W; ++r) {
    if (rcn[r]) NCKB(rt.Send(e->y_recv + roff[r] * d, (size_t)rcn[r] * d * 2, ncclUint8, r, e->comm, s));
    if (sc[r]) NCKB(rt.Recv(e->back + soff[r] * d, (size_t)sc[r] * d * 2, ncclUint8, r, e->comm, s));
  }
  NCKB(rt.GroupEnd());
  // 6. y[t] = sum_j back[pair_pos[t, j]] in j order
  return ms_ep_combine(p, e->back, e->pair_pos, T, y, stream);
}

int ms_pool_profile(ms_pool* p, int enable) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  CK(cudaSetDevice(p->device));
  if (enable && p->prof_ev.empty()) {
    p->prof_ev.resize((size_t)p->geom.n_layers * 4, nullptr);
    for (auto& e : p->prof_ev) CK(cudaEventCreate(&e));
  }
  p->profile = enable != 0;
  return MS_OK;
}

int ms_pool_timing(ms_pool* p, int layer, float* out3) {
  if (!p || !out3) return fail(MS_E_INVALID, "NULL argument");
  if (p->prof_ev.empty()) return fail(MS_E_STATE, "profiling was never enabled");
  if (layer < 0 || layer >= p->geom.n_layers) return fail(MS_E_INVALID, "layer out of range");
  cudaEvent_t* ev = &p->prof_ev[(size_t)layer * 4];
  HWAIT(event_wait_bounded(ev[3]));
  for (int i = 0; i < 3; ++i) CK(cudaEventElapsedTime(&out3[i], ev[i], ev[i + 1]));
  return MS_OK;
}

// The pool's persistent state as (device pointer, bytes) segments: the slot
// table and its counters, then (with_arena) the slot arena. Per-call scratch
// (fill lists, groups, arrival counters, which are zero between calls) is not
// part of it.
static std::vector<std::pair<void*, size_t>> state_segments(ms_pool* p, int with_arena) {
  const DevTable& t = p->tab;
  const size_t ns = (size_t)t.n_slots, nk = (size_t)t.n_keys;
  std::vector<std::pair<void*, size_t>> seg = {
      {t.key_of, 4 * ns},      {t.slot_of, 4 * nk},  {t.freq, 4 * nk},     {t.born, 8 * nk},
      {t.last_use, 8 * nk},    {t.kflags, nk},       {t.pinned, ns},       {t.pin_list, 4 * ns},
      {t.pend_list, 4 * ns},   {t.ctr, sizeof(TableCtr)}, {p->slot_class, ns}};
  if (with_arena) seg.push_back({p->arena, p->arena_bytes});
  return seg;
}

static size_t seg_round(size_t b) { return (b + 255) & ~size_t(255); }

int ms_pool_state_bytes(ms_pool* p, int with_arena, size_t* bytes) {
  if (!p || !bytes) return fail(MS_E_INVALID, "NULL argument");
  size_t n = 0;
  for (const auto& sg : state_segments(p, with_arena)) n += seg_round(sg.second);
  *bytes = n;
  return MS_OK;
}

static int copy_state(ms_pool* p, void* buf, int with_arena, cudaStream_t s, bool save) {
  if (!buf || (reinterpret_cast<uintptr_t>(buf) & 255u))
    return fail(MS_E_INVALID, "the state buffer must be a 256-byte aligned device pointer");
  CK(cudaSetDevice(p->device));
  // no prefetch fill may still be writing the arena or the table's slots
  if (int rc = join_side(p, s)) return rc;
  uint8_t* b = static_cast<uint8_t*>(buf);
  for (const auto& sg : state_segments(p, with_arena)) {
    if (save) CK(cudaMemcpyAsync(b, sg.first, sg.second, cudaMemcpyDeviceToDevice, s));
    else CK(cudaMemcpyAsync(sg.first, b, sg.second, cudaMemcpyDeviceToDevice, s));
    b += seg_round(sg.second);
  }
  return MS_OK;
}

int ms_pool_save_state(ms_pool* p, void* dev_buf, int with_arena, void* stream) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  return copy_state(p, dev_buf, with_arena, static_cast<cudaStream_t>(stream), true);
}

int ms_pool_load_state(ms_pool* p, const void* dev_buf, int with_arena, void* stream) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  p->used = true;
  return copy_state(p, const_cast<void*>(dev_buf), with_arena, static_cast<cudaStream_t>(stream),
                    false);
}

int ms_pool_set_precision(ms_pool* p, int n_classes, const ms_prec* classes,
                          const uint8_t* class_of_key) {
  if (!p || !classes || !class_of_key) return fail(MS_E_INVALID, "NULL argument");
  if (n_classes < 1 || n_classes > MS_MAX_CLASSES)
    return fail(MS_E_INVALID, "n_classes must be in [1, %d]", MS_MAX_CLASSES);
  if (p->used)
    return fail(MS_E_STATE, "precision classes must be set before the first slot fill");
  const ms_geom& g = p->geom;
  const int D = g.d_model, F = g.d_ff;
  ClassTab t{};
  t.n = n_classes;
  for (int i = 0; i < n_classes; ++i) {
    const ms_prec& c = classes[i];
    if (c.bits != 2 && c.bits != 3 && c.bits != 4 && c.bits != 8)
      return fail(MS_E_INVALID, "class %d: bits must be 2, 3, 4 or 8 (got %d)", i, c.bits);
    if (c.scale_fmt != MS_SCALE_BF16 && c.scale_fmt != MS_SCALE_FP8)
      return fail(MS_E_INVALID, "class %d: unknown scale format %d", i, c.scale_fmt);
    if (c.payload_bytes <= 0 || c.payload_bytes > g.blob_bytes)
      return fail(MS_E_INVALID, "class %d: payload_bytes must be in (0, blob_bytes]", i);
    const int esz = c.scale_fmt == MS_SCALE_FP8 ? 1 : 2;
    for (int pr = 0; pr < 3; ++pr) {
      const int n_out = pr < 2 ? F : D, n_in = pr < 2 ? D : F, G = n_in / 64;
      const long long sz[6] = {(long long)n_out * code_row_bytes(n_in, c.bits), (long long)n_out * G * esz,
                               (long long)n_out * G * esz, (long long)n_out * 2, n_out, n_out};
      const bool need[6] = {true, true, true, g.proj_bias != 0, esz == 1, esz == 1};
      for (int pt = 0; pt < 6; ++pt) {
        const long long off = c.comp_offset[pr][pt];
        if (!need[pt]) continue;
        if (off < 0 || off % 16 || off + sz[pt] > c.payload_bytes)
          return fail(MS_E_INVALID, "class %d: component [%d][%d] at %lld (+%lld) is not a 16-byte "
                      "aligned range inside the payload", i, pr, pt, off, sz[pt]);
        t.c[i].off[pr][pt] = off;
      }
    }
    t.c[i].bits = c.bits;
    t.c[i].fmt = c.scale_fmt;
  }
  for (long long k = 0; k < p->n_keys; ++k)
    if (class_of_key[k] >= n_classes)
      return fail(MS_E_INVALID, "class_of_key[%lld] = %d is not a class", k, (int)class_of_key[k]);
  CK(cudaSetDevice(p->device));
  // one class that is the geometry's own blob keeps the uniform kernels
  bool same = n_classes == 1 && classes[0].bits == 4 && classes[0].scale_fmt == MS_SCALE_BF16;
  for (int pr = 0; pr < 3 && same; ++pr)
    for (int pt = 0; pt < 4 && same; ++pt)
      if (g.comp_offset[pr][pt] >= 0 && classes[0].comp_offset[pr][pt] != g.comp_offset[pr][pt]) same = false;
  if (same) {
    default_classes(p);
    return MS_OK;
  }
  if (p->wide)
    if (int rc = encode_class_maps(p, t)) return rc;
  CK(cudaMemcpy(p->class_of_key, class_of_key, (size_t)p->n_keys, cudaMemcpyHostToDevice));
  p->h_class_of_key.assign(class_of_key, class_of_key + p->n_keys);
  p->ctab = t;
  for (int i = 0; i < n_classes; ++i) p->cls_bytes[i] = classes[i].payload_bytes;
  p->mixed = true;
  return MS_OK;
}

int ms_pool_selftest_wait(ms_pool* p, long long limit_ns, void* stream) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  if (limit_ns <= 0 || limit_ns > 2000000000LL)
    return fail(MS_E_INVALID, "limit_ns must be in (0, 2e9]");
  CK(cudaSetDevice(p->device));
  CK(launch_wait_selftest((unsigned long long)limit_ns, &p->tab.ctr->status,
                          static_cast<cudaStream_t>(stream)));
  return MS_OK;
}

int ms_kernel_arch(int device, int* binary_version) {
  if (!binary_version) return fail(MS_E_INVALID, "binary_version is NULL");
  int ndev = 0;
  CK(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return fail(MS_E_INVALID, "device %d out of range", device);
  CK(cudaSetDevice(device));
  cudaFuncAttributes attr{};
  CK(route_step_attributes(&attr));
  *binary_version = attr.binaryVersion;
  return MS_OK;
}

int ms_block_debug(ms_pool* p, const int32_t** inds, const void** scores, const int32_t** slots) {
  if (!p) return fail(MS_E_INVALID, "NULL pool");
  if (inds) *inds = p->inds;
  if (scores) *scores = p->scores;
  if (slots) *slots = p->pair_slot;
  return MS_OK;
}

}  // extern "C"
