// Kernel argument structures and launchers (host <-> device boundary inside
// libmoestream; not part of the public C ABI).
#pragma once
#include <cuda.h>   // CUtensorMap

#include "ms_common.cuh"
#include "prec.cuh"

#ifndef MS_MAX_DEPTHS
#define MS_MAX_DEPTHS 4
#endif
#define MS_MAX_REQ 256
#define MS_MLP_MAX_PAIRS 2048

struct ms_geom;   // include/moestream.h

namespace ms {

// Checks a geometry for every entry point that takes one: model and
// quantisation, shapes, and every component the kernels read inside the
// blob (offset + size <= blob_bytes) and 16-byte aligned. Returns MS_OK or
// MS_E_INVALID with the reason written to msg.
int validate_geom(const ::ms_geom* g, char* msg, size_t n);

// True when the decode expert kernels (launch_expert) handle this shape.
bool expert_shape_ok(int model, int d_model, int d_ff);

struct RouteArgs {
  Geo geo;
  const uint16_t* x;          // bf16 [T, d_model]
  int T;
  const uint16_t* w_r;        // bf16 [E, d_model]
  const uint16_t* b_r;        // bf16 [E] or null
  int n_pred;                 // prefetch targets (0..MS_MAX_DEPTHS)
  const uint16_t* w_p[MS_MAX_DEPTHS];
  const uint16_t* b_p[MS_MAX_DEPTHS];
  int pred_layer[MS_MAX_DEPTHS];   // -1: past the last layer, no prefetch
  int kp;                     // top_k * pf_widen
  float* logits;              // [T, E*(1+n_pred)]
  unsigned* ticket;
  int* inds;                  // [T, k]
  uint16_t* scores;           // [T, k] bf16
  float* scores_f;            // [T, k]
  int* pred_out;              // [T, kp] (depth 0) or null
  __half* xfrag;              // frag layout of x, or null
  float* xsum;
  int do_pool;
  DevTable tab;
  int layer;
  int do_groups;
  Groups grp;
  int* pair_slot;             // [T, k] or null
  int2* pf_ring;              // this call's half of the prefetch-fill ring, or null
  int* pf_cnt;                // its fill count
  // fused post-attention norm: x is the residual stream h and the block
  // routes rms_norm(h) * norm_w (null: x is the block input as it is)
  const uint16_t* norm_w;     // bf16 [d_model]
  float norm_eps;
};

struct PoolReq {
  int op;                     // 0 prefetch, 1 acquire
  int layer;
  int n;
  int experts[MS_MAX_REQ];
};

struct FillArgs {
  const uint8_t* store;       // device-mapped pinned host store
  uint8_t* arena;
  long long blob;
  long long store_keys;       // blobs present in the store
  const int2* fills;
  int max_fills;
  TableCtr* ctr;
  int acquire_only;           // fills[n_fill_pf, n_fill) only: the prefetch part runs elsewhere
  const int2* ring;           // else: this list of ring_cnt fills (a prefetch-fill ring half)
  const int* ring_cnt;
  int* ring_err;              // error sink of ring fills
  int pdl;                    // launched as a programmatic dependent of the route step
  const void* l2_next;        // bytes the next block call's route step will read first
  unsigned l2_next_bytes;     // (a multiple of 16), prefetched into L2; 0 for none
  // precision classes (null class_of_key: one class, whole blobs)
  const uint8_t* class_of_key;  // [n_keys]
  uint8_t* slot_class;          // [n_slots]: written with each fill
  int cls_chunks[MS_MAX_CLASSES];   // 16 KiB chunks a fill of the class copies
};

struct MlpPrepArgs {
  const uint16_t* x;
  int T, k, d_model, n_slots;
  const int* slots;           // [T, k]
  int* keys;                  // [T, k] scratch: slot, or n_slots when invalid
  TableCtr* ctr;              // status sink for invalid slots
  __half* xfrag;
  float* xsum;
  Groups grp;
};

struct ExpArgs {
  Geo geo;
  const uint8_t* arena;
  Groups grp;
  int T;
  const __half* xfrag;        // [T][d_model/64][64]
  const float* xsum;          // [T][d_model/64][2]
  __half* hfrag;              // [P][d_ff/64][64]
  float* hpart;               // [P][d_ff/16][2]
  float* ypart;               // [P][d_model]
  const float* scores;        // [P]
  unsigned* cnt;              // [d_model/16]
  uint16_t* y;                // bf16 [T, d_model]
  int* status;                // sticky pool status (bounded waits report here)
  const uint8_t* slot_class;  // [n_slots] precision class of each slot's blob (mixed pools)
  const uint16_t* resid;      // bf16 [T, d_model] added to the output (fused residual), or null
  // k of a one-token block call, whose route step leaves exactly k groups
  // (the token's distinct experts): k_down then combines within clusters of
  // k CTAs; 0 for the general arrival-counter combine
  int cl_k;
};

// ------------------------------------------------ wide batches (prefill)
// A token tile of the grouped GEMM (at most 256 rows): rows [row0, row0 +
// rows) of the expert-ordered pair list, all routed to group g.
struct GemmTile {
  int g, row0, rows;
  int slot;                   // the group's slot, -1 when the pool could not place it
};

struct WideArgs {
  int* cnt_e;                 // [256] pairs per expert; zero between calls
  unsigned* pmask;            // [MS_MAX_DEPTHS][8] predicted experts; zero between calls
  int* cursor;                // [256] per-group scatter cursors (zeroed by the router)
  GemmTile* tiles;            // [max_tiles]
  int* n_tiles;
  int max_tiles;
};

struct ScatterArgs {
  const uint16_t* x;          // bf16 [T, d]
  int T, k, d;
  const int* inds;            // [T, k] experts
  const float* scores_f;      // [T, k]
  Groups grp;
  int* cursor;
  uint16_t* xperm;            // bf16 [P_pad, d], expert order, k-permuted columns
  float* perm_score;          // [P_pad]
  int* inv;                   // [T, k] pair -> row of xperm
  int* pair_slot;             // [T, k] or null
  int* status;                // sticky pool status (ST_E_RANGE for x beyond fp16)
};

struct GemmArgs {
  int model;
  const uint8_t* arena;
  long long blob;
  long long off[3][4];
  int K;                      // reduction length: d_model (phase 0) or d_ff (phase 1)
  int n_out;                  // output rows of the projection: d_ff (phase 0) or d_model
  const GemmTile* tiles;
  const int* n_tiles;
  uint16_t* H;                // phase 0 output, fp16 [P_pad, d_ff], k-permuted columns
  uint16_t* Y;                // phase 1 output, bf16 [P_pad, d_model], score-weighted
  int ld_out;
  const float* perm_score;
  int* status;
  const uint8_t* slot_class;  // mixed pools: class of each slot, and the classes
  ClassTab C;
};

// Code-tile tensor maps of the grouped GEMM, per precision class: phase 0
// w[0] gate, w[1] up; phase 1 w[0] down.
struct GemmMaps {
  CUtensorMap w[2][MS_MAX_CLASSES];
};

struct CombineArgs {
  const uint16_t* Y;          // [P_pad, d]
  const int* inv;             // [T, k]
  uint16_t* y;                // bf16 [T, d]
  int T, k, d;
  const uint16_t* resid;      // bf16 [T, d] added to the output (fused residual), or null
};

// rms_norm(h) * w, bf16 [T, d] (the fused block's input on the wide path).
cudaError_t launch_rmsnorm(const uint16_t* h, const uint16_t* w, float eps, int T, int d, uint16_t* out,
                           cudaStream_t s);

// ms_expert_mlp on a wide batch: pairs grouped by the slot they read.
struct MlpWideArgs {
  const int* slots;           // [P] caller's slot per pair
  int P, n_slots;
  int* keys;                  // [P] scratch: the slot, or n_slots when it is invalid
  int* cnt;                   // [n_slots + 1] pairs per key; zero between calls
  int* status;                // sticky pool status (MS_E_INVALID for a bad slot)
  Groups grp;
  WideArgs w;
};

// Expert-parallel dispatch: token/expert pairs packed by destination rank.
struct EpPackArgs {
  const uint16_t* x;          // bf16 [T, d]
  int T, k, d;
  const int* inds;            // [T, k] global expert ids
  const uint16_t* scores;     // bf16 [T, k]
  int world, e_local;         // without a placement: rank r owns experts [r*e_local, (r+1)*e_local)
  const int* placement;       // or [E][1 + 2*max_rep]: n_rep, then (rank, slot) per replica
  int max_rep;
  uint16_t* send_x;           // bf16 [T * k, d], destination-major
  int* send_meta;             // [T * k][2]: slot on the destination, score (f32 bits)
  int* counts;                // [world] pairs per destination (zeroed before)
  int* cursor;                // [world] (zeroed before)
  int* pair_pos;              // [T * k] row of each pair in send_x
};

cudaError_t launch_mlp_wide_prep(const MlpWideArgs& a, int sms, cudaStream_t s);
cudaError_t launch_ep_pack(const EpPackArgs& a, int sms, cudaStream_t s);
cudaError_t launch_route_step(const RouteArgs& a, int grid, cudaStream_t s);
// One CTA waits (bounded, limit_ns) on an mbarrier whose phase never
// completes and records MS_E_TIMEOUT in *status.
cudaError_t launch_wait_selftest(unsigned long long limit_ns, int* status, cudaStream_t s);
// Attributes of the route-step kernel (its binaryVersion is the SASS target).
cudaError_t route_step_attributes(cudaFuncAttributes* attr);
cudaError_t route_prefer_shared();
cudaError_t launch_route_wide(const RouteArgs& a, const WideArgs& w, cudaStream_t s);
cudaError_t launch_scatter(const ScatterArgs& a, int grid, cudaStream_t s);
// Persistent grouped GEMM over at most max_items (token tile, feature tile)
// items, one CTA per SM (sms).
// mixed: the pool has precision classes (a.C, a.slot_class; maps.w per class),
// else every slot is the geometry's 4-bit bf16 blob (maps.w[.][0]).
cudaError_t launch_gemm(int phase, const CUtensorMap& tX, const GemmMaps& maps, const GemmArgs& a,
                        bool mixed, int max_items, int sms, cudaStream_t s);
cudaError_t launch_combine(const CombineArgs& a, int grid, cudaStream_t s);
// Tensor maps of the grouped GEMM. 0 on success.
int encode_act_map(CUtensorMap* m, const void* base, int K, long long rows);
// Weight codes of one projection across all slots, as bytes [n_slots]
// [rows_out][row_bytes], in boxes of box_bytes x box_rows x 1 slot.
int encode_codes_map(CUtensorMap* m, const void* base, int row_bytes, int rows_out, int n_slots,
                     long long blob, int box_bytes, int box_rows);
// Bytes per staged row of a GEMM K tile (64 codes) of a class: 8*bits,
// except 3 bits, whose 24-byte tile is read as the 32 bytes from the
// 16-byte boundary at or below it.
__host__ __device__ inline int gemm_tile_row_bytes(int bits) { return bits == 3 ? 32 : 8 * bits; }
// Token rows per GEMM tile.
constexpr int GEMM_TILE_ROWS = 128;
cudaError_t launch_pool_op(const DevTable& t, const PoolReq& r, int* slots_out, int* st,
                           cudaStream_t s);
cudaError_t launch_fill(const FillArgs& f, int grid, cudaStream_t s);
cudaError_t launch_mlp_prep(const MlpPrepArgs& a, cudaStream_t s);
// The decode expert kernels. maps: null, or the tensor maps of the gate, up
// and down weight rows over the arena (encode_rows_map with 16, 16 and the
// down kernel's rows per tile), which replace the per-row copies.
cudaError_t launch_expert(const ExpArgs& a, int max_groups, cudaStream_t s,
                          const CUtensorMap* maps = nullptr);
// The decode expert kernels of a pool with precision classes (expert_mx.cu).
cudaError_t launch_expert_mx(const ExpArgs& a, const ClassTab& C, int max_groups, cudaStream_t s);
// Rows per tensor-map box of the down kernel for this shape (0: no map path).
int expert_down_rows(int model, int d_model, int d_ff);
int encode_rows_map(CUtensorMap* m, const void* base, int row_bytes, int rows_out, int n_slots,
                    long long blob, int box_rows);

// Message returned by the next ms_last_error() on this thread.
void set_error_message(const char* msg);

}  // namespace ms
