// Batched, device-resident optimizer step: every registered tensor is stepped
// by one enqueue of a handful of kernels (optionally one CUDA graph launch).
// This replaces the per-tensor optim_step_weight calls of one training step
// (crates/mmn-models/src/chatbot.rs:208-227) with identical arithmetic:
// tensors keep the reference's call order, which fixes each AdamW tensor's
// step count t (crates/mmn-optim/src/lib.rs:41-43).
#include <algorithm>
#include <array>
#include <climits>
#include <cstring>
#include <unordered_set>

#include <nvtx3/nvToolsExt.h>

#include "capi_internal.cuh"
#include "elementwise.cuh"
#include "ns_engine.cuh"
#include "ns_gemm.cuh"

using namespace mmn;

namespace {

int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

// NVTX range over one host-side phase (a no-op unless a profiler is attached),
// so that a timeline shows which part of the step enqueued which kernels.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

struct ShardTensor {
  int64_t numel = 0;
  int route = MMN_ROUTE_ADAMW;  // resolved route
  int rows = 0, cols = 0;       // Muon matrices
};

struct ShardPlan {
  std::vector<int64_t> off;  // element offset in the tensor's arena
  std::vector<int> t_offset; // AdamW: 1-based position among the step's AdamW calls
  std::vector<int> owner;    // Muon: owner rank; AdamW: -1
  int n_adamw = 0;
  int64_t a_used4 = 0, a_region4 = 0;  // AdamW arena: used float4s, float4s per rank
  int64_t m_region = 0;                // Muon arena: elements per rank region
};

// Layout of both arenas and the ownership of every tensor.
//  - AdamW tensors keep the registration (= reference call) order, each padded
//    to 4 elements; the arena is cut into world_size equal 256-byte-aligned
//    ranges, rank r stepping range r.
//  - Muon matrices go whole to a rank by longest-processing-time bin packing
//    on their Newton-Schulz flops (ties to the lower rank), and are stored
//    grouped by owner so each rank's matrices form one equal-size region,
//    largest first inside it.
// The plan depends only on the shapes, routes, world size and step count, so
// every rank computes the same plan without communicating.
void make_shard_plan(const std::vector<ShardTensor>& ts, int world, int ns_steps, ShardPlan* p) {
  const size_t n = ts.size();
  p->off.assign(n, 0);
  p->t_offset.assign(n, 0);
  p->owner.assign(n, -1);
  int64_t off4 = 0;
  for (size_t i = 0; i < n; ++i) {
    if (ts[i].route != MMN_ROUTE_ADAMW) continue;
    p->off[i] = off4 * 4;
    p->t_offset[i] = ++p->n_adamw;
    off4 += (ts[i].numel + 3) / 4;
  }
  p->a_used4 = off4;
  p->a_region4 = align_up((off4 + world - 1) / world, 16);
  std::vector<size_t> muon;
  for (size_t i = 0; i < n; ++i)
    if (ts[i].route == MMN_ROUTE_MUON) muon.push_back(i);
  auto cost = [&](size_t i) {
    const double a = std::min(ts[i].rows, ts[i].cols), b = std::max(ts[i].rows, ts[i].cols);
    return (double)std::max(ns_steps, 1) * (4.0 * a * a * b + 2.0 * a * a * a) + 64.0 * a * b;
  };
  std::vector<size_t> order = muon;
  std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) { return cost(a) > cost(b); });
  std::vector<double> load((size_t)world, 0.0);
  for (size_t i : order) {
    int best = 0;
    for (int r = 1; r < world; ++r)
      if (load[r] < load[best]) best = r;
    p->owner[i] = best;
    load[best] += cost(i);
  }
  // Inside a region the matrices run by cost, largest first, equal shapes
  // together (oriented, so a matrix and its transpose share a Newton-Schulz
  // batch), then registration order.
  auto shape_key = [&](size_t i) {
    return std::make_pair(std::min(ts[i].rows, ts[i].cols), std::max(ts[i].rows, ts[i].cols));
  };
  std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) {
    const double ca = cost(a), cb = cost(b);
    if (ca != cb) return ca > cb;
    return shape_key(a) < shape_key(b);
  });
  std::vector<int64_t> used((size_t)world, 0);
  for (size_t i : order) {
    p->off[i] = used[p->owner[i]];
    used[p->owner[i]] = align_up(used[p->owner[i]] + ts[i].numel, 64);
  }
  p->m_region = 64;
  for (int r = 0; r < world; ++r) p->m_region = std::max(p->m_region, used[r]);
  for (size_t i : muon) p->off[i] += (int64_t)p->owner[i] * p->m_region;
}

}  // namespace

extern "C" int mmn_optim_plan(const int64_t* shapes, const int* ndims, const int* routes, int n,
                              int use_hybrid, int ns_steps, int world_size, int* owner,
                              int64_t* offset, int64_t* adamw_region, int64_t* muon_region) {
  if (n < 0 || (n > 0 && (!shapes || !ndims || !routes)) || world_size < 1 || ns_steps < 0)
    return fail(MMN_E_INVALID, "bad plan arguments");
  std::vector<ShardTensor> ts((size_t)n);
  const int64_t* sp = shapes;
  for (int i = 0; i < n; ++i) {
    int rc;
    const int64_t numel = shape_numel(sp, ndims[i], &rc);
    if (rc != MMN_OK) return rc;
    int route = routes[i];
    if (route != MMN_ROUTE_AUTO && route != MMN_ROUTE_MUON && route != MMN_ROUTE_ADAMW)
      return fail(MMN_E_INVALID, "unknown route");
    if (!use_hybrid)
      route = MMN_ROUTE_ADAMW;
    else if (route == MMN_ROUTE_AUTO)
      route = mmn_hybrid_classify_param(sp, ndims[i]);
    ts[i].numel = numel;
    ts[i].route = route;
    if (route == MMN_ROUTE_MUON) {
      if (ndims[i] != 2 || sp[0] < 1 || sp[1] < 1 || sp[0] > (1 << 30) || sp[1] > (1 << 30))
        return fail(MMN_E_SHAPE, "Muon tensors must be 2-D");
      ts[i].rows = (int)sp[0];
      ts[i].cols = (int)sp[1];
    }
    sp += ndims[i];
  }
  ShardPlan p;
  make_shard_plan(ts, world_size, ns_steps, &p);
  for (int i = 0; i < n; ++i) {
    if (owner) owner[i] = p.owner[i];
    if (offset) offset[i] = p.off[i];
  }
  if (adamw_region) *adamw_region = p.a_region4 * 4;
  if (muon_region) *muon_region = p.m_region;
  return MMN_OK;
}

struct mmn_optim {
  Ctx ctx;
  mmn_optim_config cfg;
  BiasTable bc;
  bool finalized = false;
  bool finalize_failed = false;  // a failed finalize leaves a half-built layout
  // reduce_grads / scan_shard handles: the grads of the coming step went
  // through mmn_optim_reduce_grads / mmn_optim_scan_grads
  bool grads_ready = false;

  struct Slot {
    uint64_t id = 0;
    std::vector<int64_t> shape;
    int64_t numel = 0;
    int route = MMN_ROUTE_ADAMW;  // resolved: MMN_ROUTE_MUON or MMN_ROUTE_ADAMW
    int64_t off = 0;              // element offset in its arena
    int t_offset = 0;             // AdamW: 1-based call position in a step
    int rows = 0, cols = 0;       // Muon
    int owner = -1;               // Muon owner rank
  };
  std::vector<Slot> slots;
  std::unordered_set<uint64_t> ids;

  // AdamW arena (fp32 p/m/v, grads in grad_dtype, optional bf16 shadow)
  int64_t a_used4 = 0, a_region4 = 0, a_total4 = 0;
  float *ap = nullptr, *am = nullptr, *av = nullptr;
  void* ag = nullptr;
  __nv_bfloat16* ap16 = nullptr;
  AdamwSeg* d_segs = nullptr;
  int* d_chunk_seg = nullptr;
  int n_adamw = 0;

  // Muon arena
  int64_t m_region = 0, m_total = 0;
  float *mp = nullptr, *mvel = nullptr;
  void* mg = nullptr;
  __nv_bfloat16* mp16 = nullptr;
  std::vector<NsClass> classes;
  std::vector<MuonMat> mats;  // owned by this rank
  MuonMat* d_mats = nullptr;
  MuonClassPtr *d_cls_in = nullptr, *d_cls_out = nullptr;
  float* d_partials = nullptr;
  float* d_norms = nullptr;
  NsApply* d_apply = nullptr;   // per owned matrix, indexed like the norms
  std::vector<int64_t> chunk_begin, chunk_end;  // Muon arena range of every NS chunk
  int norm_cluster = 1;                       // CTAs per matrix of the norm launch (all chunks)
  int norm_scalar_rows = 0;                     // a matrix's oriented rows are not 8-element groups
  std::vector<int> chunk_norm_cluster;          // the same for one chunk's launch
  std::vector<int> chunk_mat0, chunk_tile0;     // first matrix / 64x64 tile of every
                                                // chunk (one past the end appended)
  std::vector<std::vector<int>> chunk_slots;    // slots of every chunk
  // Order of the step's jobs: >= 0 is NS chunk k, < 0 is AdamW part -1 - p
  // (host-memory steps step the AdamW range in parts; the device step in one
  // launch). Compute-heavy and copy-heavy chunks alternate.
  std::vector<int> jobs;
  struct Piece {
    int slot;
    int64_t lo, hi;  // element range of the slot
  };
  std::vector<int64_t> apart_begin4, apart_end4;
  std::vector<std::vector<Piece>> apart_pieces;  // AdamW slots' ranges inside every part
  // host-memory steps: grads in and params out on two copy streams, per job
  cudaStream_t h2d = nullptr, d2h = nullptr;
  std::vector<cudaEvent_t> h2d_ev;              // [j] job j's grads landed, back() all grads
  std::vector<cudaEvent_t> apart_ev;            // AdamW part p stepped
  cudaEvent_t d2h_done = nullptr;
  // peer exchange: IPC mappings of the other ranks' parameter arenas (fp32,
  // or the bf16 copies when they are kept), filled by copy engines per chunk
  int n_peers = 0;
  void* peer_a[8] = {};
  void* peer_m[8] = {};
  std::vector<void*> peer_maps;
  // data-parallel grad reduction: every rank's grad arenas and skip flag in
  // rank order (this rank's own at [rank]), and this rank's Muon range
  const void* rank_ga[8] = {};
  const void* rank_gm[8] = {};
  int* rank_skip[8] = {};
  bool reduce_ready = false;
  int64_t m_own_begin = 0, m_own_end = 0;
  // one transfer stream per peer (and its end-of-step event): no peer's push
  // waits behind another's
  cudaStream_t xfer[mmn::kMaxRanks - 1] = {};
  cudaEvent_t xfer_done[mmn::kMaxRanks - 1] = {};
  std::vector<cudaEvent_t> chunk_ev;
  cudaEvent_t adamw_ev = nullptr;
  std::vector<int> cls_base;    // first norm / apply slot of every class
  int total_tiles = 0;
  double ns_flops = 0.0;
  int64_t n_params = 0, n_adamw_params = 0, n_muon_params = 0;

  // device step state
  long long* d_step = nullptr;
  int* d_skip = nullptr;
  float* d_scale = nullptr;
  int* d_good = nullptr;
  int* d_skipped = nullptr;

  cudaStream_t work = nullptr;  // the step's own stream, event-joined to ctx.stream
  cudaStream_t side = nullptr;  // AdamW runs here, overlapping the Newton-Schulz GEMMs
  cudaEvent_t in_ev = nullptr, out_ev = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  cudaGraphExec_t graph = nullptr;
  float graph_divisor = 0.0f;
  bool timing = false;
  // per-step phase events while timing is on: one set of 9 per step (up to
  // kTimedSteps, then the sets are reused), averaged by mmn_optim_last_timing
  static constexpr size_t kTimedSteps = 4096;
  std::vector<std::array<cudaEvent_t, 9>> ev_sets;
  size_t ev_used = 0;
  std::vector<void*> allocs;

  int dalloc(void** p, size_t bytes) {
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
    allocs.push_back(*p);
    e = cudaMemset(*p, 0, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemset");
    return MMN_OK;
  }
};

extern "C" mmn_optim_config mmn_optim_config_default(void) {
  mmn_optim_config c;
  memset(&c, 0, sizeof(c));
  c.adamw = mmn_adamw_config_default();
  c.muon = mmn_muon_config_default();
  c.use_hybrid = 1;
  c.ns_mode = MMN_NS_REFERENCE;
  c.fresh_state = 0;
  c.grad_dtype = MMN_DTYPE_F32;
  c.bf16_param_shadow = 0;
  c.loss_scaling = 0;
  c.loss_scale_init = 65536.0f;
  c.growth_interval = 2000;
  c.rank = 0;
  c.world_size = 1;
  c.use_graph = 1;
  c.reduce_grads = 0;
  c.scan_shard = 0;
  return c;
}

extern "C" int mmn_optim_create(const mmn_optim_config* cfg, int device, void* stream,
                                mmn_optim_t** out) {
  if (!out) return fail(MMN_E_INVALID, "out is null");
  *out = nullptr;
  mmn_optim_config c = cfg ? *cfg : mmn_optim_config_default();
  if (c.world_size < 1 || c.rank < 0 || c.rank >= c.world_size)
    return fail(MMN_E_INVALID, "rank / world_size out of range");
  if (c.ns_mode < MMN_NS_REFERENCE || c.ns_mode > MMN_NS_FP32)
    return fail(MMN_E_INVALID, "unknown ns_mode");
  if (c.grad_dtype != MMN_DTYPE_F32 && c.grad_dtype != MMN_DTYPE_BF16)
    return fail(MMN_E_INVALID, "grad_dtype must be f32 or bf16");
  if (c.muon.ns_steps < 0) return fail(MMN_E_INVALID, "ns_steps must be >= 0");
  if (c.loss_scaling && !(c.loss_scale_init > 0.0f)) return fail(MMN_E_INVALID, "loss scale <= 0");
  if (c.scan_shard && (!c.loss_scaling || c.world_size < 2 || c.reduce_grads))
    return fail(MMN_E_INVALID,
                "scan_shard needs loss_scaling, world_size > 1 and reduce_grads = 0");
  auto* h = new mmn_optim();
  h->cfg = c;
  int rc = h->ctx.init(device, stream);
  if (rc == MMN_OK) {
    DeviceGuard g(device);
    rc = h->bc.build(c.adamw.beta1, c.adamw.beta2);
  }
  if (rc != MMN_OK) {
    h->ctx.release();
    delete h;
    return rc;
  }
  *out = h;
  return MMN_OK;
}

extern "C" int mmn_optim_destroy(mmn_optim_t* h) {
  if (!h) return MMN_OK;
  DeviceGuard g(h->ctx.device);
  cudaStreamSynchronize(h->ctx.stream);
  if (h->graph) cudaGraphExecDestroy(h->graph);
  for (auto& c : h->classes) ns_class_free(c);
  for (void* p : h->peer_maps) cudaIpcCloseMemHandle(p);
  for (void* p : h->allocs) cudaFree(p);
  for (auto& set : h->ev_sets)
    for (auto e : set)
      if (e) cudaEventDestroy(e);
  if (h->fork) cudaEventDestroy(h->fork);
  if (h->join) cudaEventDestroy(h->join);
  if (h->side) cudaStreamDestroy(h->side);
  for (auto st : h->xfer)
    if (st) cudaStreamDestroy(st);
  if (h->h2d) cudaStreamDestroy(h->h2d);
  if (h->d2h) cudaStreamDestroy(h->d2h);
  for (auto e : h->chunk_ev)
    if (e) cudaEventDestroy(e);
  for (auto e : h->h2d_ev)
    if (e) cudaEventDestroy(e);
  for (auto e : h->apart_ev)
    if (e) cudaEventDestroy(e);
  if (h->adamw_ev) cudaEventDestroy(h->adamw_ev);
  for (auto e : h->xfer_done)
    if (e) cudaEventDestroy(e);
  if (h->d2h_done) cudaEventDestroy(h->d2h_done);
  if (h->work) cudaStreamDestroy(h->work);
  if (h->in_ev) cudaEventDestroy(h->in_ev);
  if (h->out_ev) cudaEventDestroy(h->out_ev);
  h->bc.release();
  h->ctx.release();
  delete h;
  return MMN_OK;
}

extern "C" int mmn_optim_add_param(mmn_optim_t* h, uint64_t id, const int64_t* shape, int ndim,
                                   int route, int* slot) {
  if (!h) return fail(MMN_E_INVALID, "null handle");
  if (h->finalized) return fail(MMN_E_STATE, "add_param after finalize");
  if (h->ids.count(id)) return fail(MMN_E_INVALID, "id registered twice");
  int rc;
  const int64_t numel = shape_numel(shape, ndim, &rc);
  if (rc != MMN_OK) return rc;
  if (route != MMN_ROUTE_AUTO && route != MMN_ROUTE_MUON && route != MMN_ROUTE_ADAMW)
    return fail(MMN_E_INVALID, "unknown route");
  mmn_optim::Slot s;
  s.id = id;
  s.shape.assign(shape, shape + ndim);
  s.numel = numel;
  if (!h->cfg.use_hybrid)
    s.route = MMN_ROUTE_ADAMW;  // crates/mmn-train/src/lib.rs:378: only "hybrid" uses Muon
  else if (route == MMN_ROUTE_AUTO)
    s.route = mmn_hybrid_classify_param(shape, ndim);
  else
    s.route = route;
  if (s.route == MMN_ROUTE_MUON) {
    if (ndim != 2 || shape[0] < 1 || shape[1] < 1 || shape[0] > (1 << 30) || shape[1] > (1 << 30))
      return fail(MMN_E_SHAPE, "Muon tensors must be 2-D");
    s.rows = (int)shape[0];
    s.cols = (int)shape[1];
  }
  h->ids.insert(id);
  h->slots.push_back(s);
  if (slot) *slot = (int)h->slots.size() - 1;
  return MMN_OK;
}

static int finalize_layout(mmn_optim_t* h);

extern "C" int mmn_optim_finalize(mmn_optim_t* h) {
  if (!h) return fail(MMN_E_INVALID, "null handle");
  if (h->finalized) return MMN_OK;
  if (h->finalize_failed)
    return fail(MMN_E_STATE, "an earlier finalize failed: destroy the handle and start again");
  const int rc = finalize_layout(h);
  if (rc != MMN_OK) h->finalize_failed = true;
  return rc;
}

static int finalize_layout(mmn_optim_t* h) {
  DeviceGuard g(h->ctx.device);
  const int W = h->cfg.world_size, R = h->cfg.rank;
  const int steps = h->cfg.muon.ns_steps;
  int rc;

  // ---- Layout and sharding plan (host only; shared with mmn_optim_plan).
  std::vector<ShardTensor> pts(h->slots.size());
  for (size_t i = 0; i < h->slots.size(); ++i) {
    pts[i].numel = h->slots[i].numel;
    pts[i].route = h->slots[i].route;
    pts[i].rows = h->slots[i].rows;
    pts[i].cols = h->slots[i].cols;
  }
  ShardPlan plan;
  make_shard_plan(pts, W, steps, &plan);
  std::vector<int> muon_idx;
  for (size_t i = 0; i < h->slots.size(); ++i) {
    auto& s = h->slots[i];
    s.off = plan.off[i];
    s.t_offset = plan.t_offset[i];
    s.owner = plan.owner[i];
    h->n_params += s.numel;
    if (s.route == MMN_ROUTE_MUON) {
      h->n_muon_params += s.numel;
      muon_idx.push_back((int)i);
    } else {
      h->n_adamw_params += s.numel;
    }
  }
  h->n_adamw = plan.n_adamw;
  h->a_used4 = plan.a_used4;
  h->a_region4 = plan.a_region4;
  h->a_total4 = h->a_region4 * W;
  h->m_region = plan.m_region;
  h->m_total = h->m_region * W;
  std::vector<AdamwSeg> segs;
  for (auto& s : h->slots) {
    if (s.route != MMN_ROUTE_ADAMW || s.numel == 0) continue;
    AdamwSeg sg{};
    sg.start4 = s.off / 4;
    sg.end4 = sg.start4 + (s.numel + 3) / 4;
    sg.t_offset = s.t_offset;
    segs.push_back(sg);
  }
  std::vector<int> chunk_seg((size_t)((h->a_used4 + kAdamwChunk4 - 1) / kAdamwChunk4) + 1, 0);
  for (size_t k = 0, c = 0; c < chunk_seg.size(); ++c) {
    const int64_t first = (int64_t)c * kAdamwChunk4;
    while (k + 1 < segs.size() && segs[k].end4 <= first) ++k;
    chunk_seg[c] = (int)k;
  }

  // ---- Newton-Schulz chunks over the matrices this rank owns, in arena order
  // (largest shapes first): runs of one shape, at most kNsChunk matrices and
  // kChunkElems elements each (256 MB of fp32: big enough to fill the GPU with
  // tiles, small enough that a chunk's PCIe or NVLink copy is short).
  // Chunks run one after another, so with the peer exchange each finished
  // chunk's parameters cross NVLink while the following chunks compute, and a
  // step from host memory overlaps each chunk's copies with its neighbours'
  // compute.
  constexpr int kNsChunk = 16;
  constexpr int64_t kChunkElems = int64_t(1) << 26;
  std::vector<int> owned;
  for (int i : muon_idx)
    if (h->slots[i].owner == R) owned.push_back(i);
  std::stable_sort(owned.begin(), owned.end(),
                   [&](int a, int b) { return h->slots[a].off < h->slots[b].off; });
  std::vector<std::pair<int, int>> cls_shapes;
  std::vector<int> cls_count;
  int tiles = 0;
  for (int i : owned) {
    auto& s = h->slots[i];
    const int n = std::min(s.rows, s.cols), m = std::max(s.rows, s.cols);
    if (cls_shapes.empty() || cls_shapes.back() != std::make_pair(n, m) ||
        cls_count.back() == kNsChunk ||
        s.off + s.numel - h->chunk_begin.back() > kChunkElems) {
      cls_shapes.emplace_back(n, m);
      cls_count.push_back(0);
      h->chunk_begin.push_back(s.off);
      h->chunk_end.push_back(s.off);
      h->chunk_mat0.push_back((int)h->mats.size());
      h->chunk_tile0.push_back(tiles);
      h->chunk_slots.emplace_back();
    }
    const int ci = (int)cls_shapes.size() - 1;
    h->chunk_end[ci] = s.off + s.numel;
    h->chunk_slots[ci].push_back(i);
    MuonMat mm{};
    mm.off = s.off;
    mm.rows = s.rows;
    mm.cols = s.cols;
    mm.transposed = s.rows > s.cols;
    mm.xcls = ci;
    mm.xbatch = cls_count[ci]++;
    mm.tile0 = tiles;
    tiles += ((s.rows + 63) / 64) * ((s.cols + 63) / 64);
    mm.lr_scale = h->cfg.muon.lr * sqrtf((float)s.rows / (float)s.cols);  // lib.rs:169-173
    h->mats.push_back(mm);
    h->ns_flops += (double)steps * (4.0 * n * (double)n * m + 2.0 * (double)n * n * n);
  }
  h->total_tiles = tiles;
  h->m_own_begin = (int64_t)R * h->m_region;
  h->m_own_end = h->m_own_begin;
  for (int64_t e : h->chunk_end) h->m_own_end = std::max(h->m_own_end, align_up(e, 64));
  h->chunk_mat0.push_back((int)h->mats.size());
  h->chunk_tile0.push_back(tiles);
  {
    // CTAs per matrix of the sequential-norm launches, over every chunk at
    // once (device steps) and per chunk (steps from host memory)
    auto elems = [&](const MuonMat& mm) { return (long long)mm.rows * mm.cols; };
    long long mx = 0, tot = 0;
    for (const MuonMat& mm : h->mats) {
      mx = std::max(mx, elems(mm));
      tot += elems(mm);
      if (std::max(mm.rows, mm.cols) % 8 != 0) h->norm_scalar_rows = 1;
    }
    h->norm_cluster = ref_norm_cluster(mx, tot, (int)h->mats.size(), h->ctx.num_sms);
    for (size_t k = 0; k + 1 < h->chunk_mat0.size(); ++k) {
      long long cmx = 0, ctot = 0;
      for (int i = h->chunk_mat0[k]; i < h->chunk_mat0[k + 1]; ++i) {
        cmx = std::max(cmx, elems(h->mats[i]));
        ctot += elems(h->mats[i]);
      }
      h->chunk_norm_cluster.push_back(
          ref_norm_cluster(cmx, ctot, h->chunk_mat0[k + 1] - h->chunk_mat0[k], h->ctx.num_sms));
    }
  }

  // ---- AdamW parts over this rank's range: at most kChunkElems elements each,
  // and, when the range is large, a small first and last part (2^24 elements)
  // so that a host-memory step's copies start back early and end soon after
  // the last grads land
  {
    const int64_t lo4 = std::min<int64_t>(h->a_region4 * R, h->a_used4);
    const int64_t hi4 = std::min<int64_t>(h->a_region4 * (R + 1), h->a_used4);
    const int64_t n4 = hi4 - lo4;
    constexpr int64_t kEdge4 = (int64_t(1) << 24) / 4;
    std::vector<int64_t> cuts{lo4};
    if (n4 > 4 * kEdge4) {
      const int64_t mid = n4 - 2 * kEdge4;
      const int64_t parts = (mid * 4 + kChunkElems - 1) / kChunkElems;
      for (int64_t p = 0; p <= parts; ++p) cuts.push_back(lo4 + kEdge4 + mid * p / parts);
      cuts.push_back(hi4);
    } else if (n4 > 0) {
      const int64_t parts = (n4 * 4 + kChunkElems - 1) / kChunkElems;
      for (int64_t p = 1; p <= parts; ++p) cuts.push_back(lo4 + n4 * p / parts);
    }
    for (size_t p = 0; p + 1 < cuts.size(); ++p) {
      const int64_t b4 = cuts[p], e4 = cuts[p + 1];
      h->apart_begin4.push_back(b4);
      h->apart_end4.push_back(e4);
      std::vector<mmn_optim::Piece> pcs;
      for (size_t i = 0; i < h->slots.size(); ++i) {
        const auto& sl = h->slots[i];
        if (sl.route != MMN_ROUTE_ADAMW) continue;
        const int64_t l = std::max<int64_t>(b4 * 4, sl.off) - sl.off;
        const int64_t u = std::min<int64_t>(e4 * 4, sl.off + sl.numel) - sl.off;
        if (u > l) pcs.push_back({(int)i, l, u});
      }
      h->apart_pieces.push_back(pcs);
    }
  }
  // ---- job order: chunks zipped from the most and the least flops per element
  // (4n + 2n^2/m for an n x m chunk), AdamW parts first and last and spread
  // between (a part's compute is short and runs beside the GEMMs, so it makes
  // the shortest pipeline head and tail)
  {
    const int nck = (int)cls_shapes.size();
    std::vector<int> ck(nck);
    for (int k = 0; k < nck; ++k) ck[k] = k;
    auto per_elem = [&](int k) {
      const double n = cls_shapes[k].first, m = cls_shapes[k].second;
      return 4.0 * n + 2.0 * n * n / m;
    };
    std::stable_sort(ck.begin(), ck.end(), [&](int a, int b) { return per_elem(a) > per_elem(b); });
    std::vector<int> zig;
    for (int lo = 0, hi = nck - 1, front = 1; lo <= hi; front ^= 1) zig.push_back(front ? ck[lo++] : ck[hi--]);
    if (W > 1 && zig.size() > 1) {
      // with peers, the last chunk's push is the one no compute hides: the
      // chunk with the fewest elements goes last (ties keep the later chunk,
      // so equal chunks keep their order)
      size_t small = 0;
      for (size_t i = 1; i < zig.size(); ++i)
        if (h->chunk_end[zig[i]] - h->chunk_begin[zig[i]] <=
            h->chunk_end[zig[small]] - h->chunk_begin[zig[small]])
          small = i;
      const int last = zig[small];
      zig.erase(zig.begin() + (long)small);
      zig.push_back(last);
    }
    const int P = (int)h->apart_begin4.size();
    std::vector<std::vector<int>> before(zig.size() + 1);  // AdamW parts placed before zig[i]
    for (int p = 0; p < P; ++p) {
      const size_t pos = P == 1 ? zig.size() : (size_t)((double)p * zig.size() / (P - 1) + 0.5);
      before[std::min(pos, zig.size())].push_back(-1 - p);
    }
    for (size_t i = 0; i <= zig.size(); ++i) {
      for (int j : before[i]) h->jobs.push_back(j);
      if (i < zig.size()) h->jobs.push_back(zig[i]);
    }
  }
  if (!h->mats.empty()) {
    std::string e = ns_gemm_setup();
    if (!e.empty()) return fail(MMN_E_CUDA, e);
  }
  h->classes.resize(cls_shapes.size());
  int norm_base = 0;
  std::vector<int> cls_norm0(cls_shapes.size());
  for (size_t k = 0; k < cls_shapes.size(); ++k) {
    std::string e = ns_class_init(h->classes[k], cls_shapes[k].first, cls_shapes[k].second,
                                  cls_count[k], nullptr, ns_elem_bytes(h->cfg.ns_mode),
                                  ns_planes(h->cfg.ns_mode));
    if (!e.empty()) return fail(MMN_E_OOM, e);
    cls_norm0[k] = norm_base;
    norm_base += cls_count[k];
  }
  for (auto& mm : h->mats) mm.norm_idx = cls_norm0[mm.xcls] + mm.xbatch;
  h->cls_base = cls_norm0;
  std::vector<NsApply> applies((size_t)std::max(norm_base, 1));
  for (auto& mm : h->mats) {
    applies[mm.norm_idx].off = mm.off;
    applies[mm.norm_idx].lr_scale = mm.lr_scale;
    applies[mm.norm_idx].transposed = mm.transposed;
  }

  // ---- device allocations
  const size_t gsz = h->cfg.grad_dtype == MMN_DTYPE_BF16 ? 2 : 4;
  const size_t a_el = (size_t)h->a_total4 * 4;
  if ((rc = h->dalloc((void**)&h->ap, a_el * 4)) != MMN_OK) return rc;
  if ((rc = h->dalloc((void**)&h->am, h->cfg.fresh_state ? 16 : a_el * 4)) != MMN_OK) return rc;
  if ((rc = h->dalloc((void**)&h->av, h->cfg.fresh_state ? 16 : a_el * 4)) != MMN_OK) return rc;
  if ((rc = h->dalloc(&h->ag, a_el * gsz)) != MMN_OK) return rc;
  if (h->cfg.bf16_param_shadow && (rc = h->dalloc((void**)&h->ap16, a_el * 2)) != MMN_OK) return rc;
  if ((rc = h->dalloc((void**)&h->d_segs, std::max<size_t>(segs.size(), 1) * sizeof(AdamwSeg))) != MMN_OK)
    return rc;
  if ((rc = h->dalloc((void**)&h->d_chunk_seg, chunk_seg.size() * sizeof(int))) != MMN_OK) return rc;
  const size_t m_el = (size_t)h->m_total;
  if ((rc = h->dalloc((void**)&h->mp, m_el * 4)) != MMN_OK) return rc;
  if ((rc = h->dalloc((void**)&h->mvel, m_el * 4)) != MMN_OK) return rc;
  if ((rc = h->dalloc(&h->mg, m_el * gsz)) != MMN_OK) return rc;
  if (h->cfg.bf16_param_shadow && (rc = h->dalloc((void**)&h->mp16, m_el * 2)) != MMN_OK) return rc;
  if ((rc = h->dalloc((void**)&h->d_mats, std::max<size_t>(h->mats.size(), 1) * sizeof(MuonMat))) != MMN_OK)
    return rc;
  const size_t ncls = std::max<size_t>(h->classes.size(), 1);
  if ((rc = h->dalloc((void**)&h->d_cls_in, ncls * sizeof(MuonClassPtr))) != MMN_OK) return rc;
  if ((rc = h->dalloc((void**)&h->d_cls_out, ncls * sizeof(MuonClassPtr))) != MMN_OK) return rc;
  if ((rc = h->dalloc((void**)&h->d_partials, (size_t)std::max(tiles, 1) * 4)) != MMN_OK) return rc;
  if ((rc = h->dalloc((void**)&h->d_norms, (size_t)std::max(norm_base, 1) * 4)) != MMN_OK) return rc;
  if ((rc = h->dalloc((void**)&h->d_apply, applies.size() * sizeof(NsApply))) != MMN_OK) return rc;
  if ((rc = h->dalloc((void**)&h->d_step, sizeof(long long))) != MMN_OK) return rc;
  if ((rc = h->dalloc((void**)&h->d_skip, sizeof(int))) != MMN_OK) return rc;
  if ((rc = h->dalloc((void**)&h->d_scale, sizeof(float))) != MMN_OK) return rc;
  if ((rc = h->dalloc((void**)&h->d_good, sizeof(int))) != MMN_OK) return rc;
  if ((rc = h->dalloc((void**)&h->d_skipped, sizeof(int))) != MMN_OK) return rc;

  MMN_CUDA_TRY(cudaMemcpy(h->d_segs, segs.data(), segs.size() * sizeof(AdamwSeg), cudaMemcpyHostToDevice));
  MMN_CUDA_TRY(cudaMemcpy(h->d_chunk_seg, chunk_seg.data(), chunk_seg.size() * sizeof(int),
                          cudaMemcpyHostToDevice));
  MMN_CUDA_TRY(cudaMemcpy(h->d_mats, h->mats.data(), h->mats.size() * sizeof(MuonMat),
                          cudaMemcpyHostToDevice));
  MMN_CUDA_TRY(cudaMemcpy(h->d_apply, applies.data(), applies.size() * sizeof(NsApply),
                          cudaMemcpyHostToDevice));
  std::vector<MuonClassPtr> cin(ncls), cout(ncls);
  for (size_t k = 0; k < h->classes.size(); ++k) {
    auto& c = h->classes[k];
    c.norms = h->d_norms + cls_norm0[k];  // the class reads its norms from the shared array
    cin[k].x = c.x[0];
    cin[k].bstride = (long long)c.n * c.ld_x;
    cin[k].ld = c.ld_x;
    cout[k] = cin[k];
    cout[k].x = c.x[steps % 2];
  }
  MMN_CUDA_TRY(cudaMemcpy(h->d_cls_in, cin.data(), ncls * sizeof(MuonClassPtr), cudaMemcpyHostToDevice));
  MMN_CUDA_TRY(cudaMemcpy(h->d_cls_out, cout.data(), ncls * sizeof(MuonClassPtr), cudaMemcpyHostToDevice));
  const float scale = h->cfg.loss_scale_init;
  MMN_CUDA_TRY(cudaMemcpy(h->d_scale, &scale, sizeof(float), cudaMemcpyHostToDevice));

  MMN_CUDA_TRY(cudaStreamCreateWithFlags(&h->side, cudaStreamNonBlocking));
  MMN_CUDA_TRY(cudaStreamCreateWithFlags(&h->work, cudaStreamNonBlocking));
  MMN_CUDA_TRY(cudaEventCreateWithFlags(&h->in_ev, cudaEventDisableTiming));
  MMN_CUDA_TRY(cudaEventCreateWithFlags(&h->out_ev, cudaEventDisableTiming));
  MMN_CUDA_TRY(cudaEventCreateWithFlags(&h->fork, cudaEventDisableTiming));
  MMN_CUDA_TRY(cudaEventCreateWithFlags(&h->join, cudaEventDisableTiming));
  for (int r = 0; r + 1 < h->cfg.world_size && r < mmn::kMaxRanks - 1; ++r) {
    MMN_CUDA_TRY(cudaStreamCreateWithFlags(&h->xfer[r], cudaStreamNonBlocking));
    MMN_CUDA_TRY(cudaEventCreateWithFlags(&h->xfer_done[r], cudaEventDisableTiming));
  }
  MMN_CUDA_TRY(cudaStreamCreateWithFlags(&h->h2d, cudaStreamNonBlocking));
  MMN_CUDA_TRY(cudaStreamCreateWithFlags(&h->d2h, cudaStreamNonBlocking));
  MMN_CUDA_TRY(cudaEventCreateWithFlags(&h->adamw_ev, cudaEventDisableTiming));
  MMN_CUDA_TRY(cudaEventCreateWithFlags(&h->d2h_done, cudaEventDisableTiming));
  h->chunk_ev.assign(h->chunk_begin.size(), nullptr);
  for (auto& e : h->chunk_ev) MMN_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  h->h2d_ev.assign(h->jobs.size() + 1, nullptr);
  for (auto& e : h->h2d_ev) MMN_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  h->apart_ev.assign(h->apart_begin4.size(), nullptr);
  for (auto& e : h->apart_ev) MMN_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  MMN_CUDA_TRY(cudaDeviceSynchronize());
  h->finalized = true;
  return MMN_OK;
}

static int check_slot(mmn_optim_t* h, int slot) {
  if (!h) return fail(MMN_E_INVALID, "null handle");
  if (!h->finalized) return fail(MMN_E_STATE, "finalize first");
  if (slot < 0 || slot >= (int)h->slots.size()) return fail(MMN_E_INVALID, "slot out of range");
  return MMN_OK;
}

static float* slot_param(mmn_optim_t* h, const mmn_optim::Slot& s) {
  return (s.route == MMN_ROUTE_ADAMW ? h->ap : h->mp) + s.off;
}

extern "C" int mmn_optim_slot_ptrs(mmn_optim_t* h, int slot, float** param, void** grad,
                                   void** param_bf16) {
  int rc = check_slot(h, slot);
  if (rc != MMN_OK) return rc;
  const auto& s = h->slots[slot];
  const size_t gsz = h->cfg.grad_dtype == MMN_DTYPE_BF16 ? 2 : 4;
  const bool a = s.route == MMN_ROUTE_ADAMW;
  if (param) *param = slot_param(h, s);
  if (grad) *grad = static_cast<uint8_t*>(a ? h->ag : h->mg) + (size_t)s.off * gsz;
  if (param_bf16) {
    __nv_bfloat16* b = a ? h->ap16 : h->mp16;
    *param_bf16 = b ? b + s.off : nullptr;
  }
  return MMN_OK;
}

static cudaMemcpyKind kind_in(int mem) {
  return mem == MMN_MEM_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
}
static cudaMemcpyKind kind_out(int mem) {
  return mem == MMN_MEM_HOST ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
}

extern "C" int mmn_optim_set_param(mmn_optim_t* h, int slot, const float* src, int mem) {
  int rc = check_slot(h, slot);
  if (rc != MMN_OK) return rc;
  if (!src) return fail(MMN_E_INVALID, "null src");
  DeviceGuard g(h->ctx.device);
  const auto& s = h->slots[slot];
  float* dst = slot_param(h, s);
  MMN_CUDA_TRY(cudaMemcpyAsync(dst, src, (size_t)s.numel * 4, kind_in(mem), h->ctx.stream));
  if (h->cfg.bf16_param_shadow) {
    // Keep the shadow equal to bf16(master) from the start.
    __nv_bfloat16* b = (s.route == MMN_ROUTE_ADAMW ? h->ap16 : h->mp16) + s.off;
    std::vector<__nv_bfloat16> tmp((size_t)s.numel);
    std::vector<float> hostp((size_t)s.numel);
    MMN_CUDA_TRY(cudaMemcpyAsync(hostp.data(), dst, (size_t)s.numel * 4, cudaMemcpyDeviceToHost,
                                 h->ctx.stream));
    MMN_CUDA_TRY(cudaStreamSynchronize(h->ctx.stream));
    for (size_t i = 0; i < hostp.size(); ++i) tmp[i] = __float2bfloat16_rn(hostp[i]);
    MMN_CUDA_TRY(cudaMemcpyAsync(b, tmp.data(), tmp.size() * 2, cudaMemcpyHostToDevice, h->ctx.stream));
  }
  if (mem == MMN_MEM_HOST) MMN_CUDA_TRY(cudaStreamSynchronize(h->ctx.stream));
  return MMN_OK;
}

extern "C" int mmn_optim_get_param(mmn_optim_t* h, int slot, float* dst, int mem) {
  int rc = check_slot(h, slot);
  if (rc != MMN_OK) return rc;
  if (!dst) return fail(MMN_E_INVALID, "null dst");
  DeviceGuard g(h->ctx.device);
  const auto& s = h->slots[slot];
  MMN_CUDA_TRY(cudaMemcpyAsync(dst, slot_param(h, s), (size_t)s.numel * 4, kind_out(mem),
                               h->ctx.stream));
  if (mem == MMN_MEM_HOST) MMN_CUDA_TRY(cudaStreamSynchronize(h->ctx.stream));
  return MMN_OK;
}

extern "C" int mmn_optim_set_grad(mmn_optim_t* h, int slot, const void* src, int mem) {
  int rc = check_slot(h, slot);
  if (rc != MMN_OK) return rc;
  if (!src) return fail(MMN_E_INVALID, "null src");
  DeviceGuard g(h->ctx.device);
  void* dst = nullptr;
  mmn_optim_slot_ptrs(h, slot, nullptr, &dst, nullptr);
  const size_t gsz = h->cfg.grad_dtype == MMN_DTYPE_BF16 ? 2 : 4;
  MMN_CUDA_TRY(cudaMemcpyAsync(dst, src, (size_t)h->slots[slot].numel * gsz, kind_in(mem),
                               h->ctx.stream));
  if (mem == MMN_MEM_HOST) MMN_CUDA_TRY(cudaStreamSynchronize(h->ctx.stream));
  return MMN_OK;
}

static int state_ptr(mmn_optim_t* h, int slot, int which, float** p) {
  const auto& s = h->slots[slot];
  if (which == 0 || which == 1) {
    if (s.route != MMN_ROUTE_ADAMW) return fail(MMN_E_INVALID, "m/v exist only for AdamW slots");
    if (h->cfg.fresh_state) return fail(MMN_E_STATE, "fresh_state handles keep no m/v");
    *p = (which == 0 ? h->am : h->av) + s.off;
    return MMN_OK;
  }
  if (which == 2) {
    if (s.route != MMN_ROUTE_MUON) return fail(MMN_E_INVALID, "velocity exists only for Muon slots");
    *p = h->mvel + s.off;
    return MMN_OK;
  }
  return fail(MMN_E_INVALID, "which must be 0 (m), 1 (v) or 2 (velocity)");
}

extern "C" int mmn_optim_set_state(mmn_optim_t* h, int slot, int which, const float* src, int mem) {
  int rc = check_slot(h, slot);
  if (rc != MMN_OK) return rc;
  if (!src) return fail(MMN_E_INVALID, "null src");
  float* p = nullptr;
  if ((rc = state_ptr(h, slot, which, &p)) != MMN_OK) return rc;
  DeviceGuard g(h->ctx.device);
  MMN_CUDA_TRY(cudaMemcpyAsync(p, src, (size_t)h->slots[slot].numel * 4, kind_in(mem), h->ctx.stream));
  if (mem == MMN_MEM_HOST) MMN_CUDA_TRY(cudaStreamSynchronize(h->ctx.stream));
  return MMN_OK;
}

extern "C" int mmn_optim_get_state(mmn_optim_t* h, int slot, int which, float* dst, int mem) {
  int rc = check_slot(h, slot);
  if (rc != MMN_OK) return rc;
  if (!dst) return fail(MMN_E_INVALID, "null dst");
  float* p = nullptr;
  if ((rc = state_ptr(h, slot, which, &p)) != MMN_OK) return rc;
  DeviceGuard g(h->ctx.device);
  MMN_CUDA_TRY(cudaMemcpyAsync(dst, p, (size_t)h->slots[slot].numel * 4, kind_out(mem), h->ctx.stream));
  if (mem == MMN_MEM_HOST) MMN_CUDA_TRY(cudaStreamSynchronize(h->ctx.stream));
  return MMN_OK;
}

extern "C" int mmn_optim_set_adamw_step(mmn_optim_t* h, uint64_t step) {
  if (!h || !h->finalized) return fail(MMN_E_STATE, "finalize first");
  DeviceGuard g(h->ctx.device);
  const long long v = (long long)step;
  MMN_CUDA_TRY(cudaMemcpyAsync(h->d_step, &v, sizeof(v), cudaMemcpyHostToDevice, h->ctx.stream));
  MMN_CUDA_TRY(cudaStreamSynchronize(h->ctx.stream));
  return MMN_OK;
}

extern "C" int mmn_optim_get_adamw_step(mmn_optim_t* h, uint64_t* step) {
  if (!h || !h->finalized || !step) return fail(MMN_E_STATE, "finalize first");
  DeviceGuard g(h->ctx.device);
  long long v = 0;
  MMN_CUDA_TRY(cudaMemcpyAsync(&v, h->d_step, sizeof(v), cudaMemcpyDeviceToHost, h->ctx.stream));
  MMN_CUDA_TRY(cudaStreamSynchronize(h->ctx.stream));
  *step = (uint64_t)v;
  return MMN_OK;
}

// Once `ready` has completed, copies elements [lo, hi) of a local parameter
// arena (fp32, or bf16 when the copies are kept) into the same range of every
// peer's arena (copy engines over NVLink through the IPC mappings). Each peer
// has a transfer stream of its own, so the copies to the peers may run side by
// side. (On 8 B200s this measured the same as one stream for all peers: the
// copy-engine pushes reach about 400 GB/s of egress per rank either way.)
static int copy_to_peers(mmn_optim_t* h, cudaEvent_t ready, void* local, void* const* peers,
                         int64_t lo, int64_t hi) {
  if (hi <= lo) return MMN_OK;
  const size_t es = h->cfg.bf16_param_shadow ? 2 : 4;
  const uint8_t* src = static_cast<const uint8_t*>(local) + (size_t)lo * es;
  for (int r = 0; r < h->n_peers; ++r) {
    MMN_CUDA_TRY(cudaStreamWaitEvent(h->xfer[r], ready, 0));
    MMN_CUDA_TRY(cudaMemcpyAsync(static_cast<uint8_t*>(peers[r]) + (size_t)lo * es, src,
                                 (size_t)(hi - lo) * es, cudaMemcpyDeviceToDevice, h->xfer[r]));
  }
  return MMN_OK;
}

// Host buffers of a step from host memory, indexed by slot: grads in the grad
// dtype, params fp32. A null entry skips that slot's copy.
struct HostIO {
  const void* const* grads;
  float* const* params;
};

// The elements [lo, hi) of a slot that this rank steps: a whole Muon matrix
// it owns, or the overlap of an AdamW tensor with its AdamW range. Returns
// false (lo == hi == 0) when it steps none of the slot.
static bool stepped_range(const mmn_optim_t* h, const mmn_optim::Slot& s, int64_t* lo,
                          int64_t* hi) {
  *lo = *hi = 0;
  if (s.route == MMN_ROUTE_MUON) {
    if (s.owner != h->cfg.rank) return false;
    *hi = s.numel;
    return true;
  }
  const int R = h->cfg.rank;
  const int64_t rlo = std::min<int64_t>(h->a_region4 * R, h->a_used4) * 4;
  const int64_t rhi = std::min<int64_t>(h->a_region4 * (R + 1), h->a_used4) * 4;
  const int64_t l = std::max<int64_t>(rlo, s.off) - s.off;
  const int64_t u = std::min<int64_t>(rhi, s.off + s.numel) - s.off;
  if (u <= l) return false;
  *lo = l;
  *hi = u;
  return true;
}

// Host grads[slot][lo, hi) -> the slot's device grads, on the h2d stream.
static int grad_in(mmn_optim_t* h, const HostIO* io, int i, int64_t lo, int64_t hi) {
  const auto& s = h->slots[i];
  if (!io->grads[i] || hi <= lo) return MMN_OK;
  const size_t gsz = h->cfg.grad_dtype == MMN_DTYPE_BF16 ? 2 : 4;
  uint8_t* dst = static_cast<uint8_t*>(s.route == MMN_ROUTE_ADAMW ? h->ag : h->mg) +
                 (size_t)(s.off + lo) * gsz;
  const uint8_t* src = static_cast<const uint8_t*>(io->grads[i]) + (size_t)lo * gsz;
  MMN_CUDA_TRY(cudaMemcpyAsync(dst, src, (size_t)(hi - lo) * gsz, cudaMemcpyHostToDevice, h->h2d));
  return MMN_OK;
}

// Device params of slot i, elements [lo, hi) -> host params[slot], on the d2h stream.
static int param_out(mmn_optim_t* h, const HostIO* io, int i, int64_t lo, int64_t hi) {
  if (!io->params[i] || hi <= lo) return MMN_OK;
  MMN_CUDA_TRY(cudaMemcpyAsync(io->params[i] + lo, slot_param(h, h->slots[i]) + lo,
                               (size_t)(hi - lo) * 4, cudaMemcpyDeviceToHost, h->d2h));
  return MMN_OK;
}

#define MMN_TRY_RC(x)            \
  do {                           \
    const int rc_ = (x);         \
    if (rc_ != MMN_OK) return rc_; \
  } while (0)

// Enqueues the whole step on the handle's work stream: AdamW forked onto a
// side stream so it overlaps the Newton-Schulz GEMMs, the Muon matrices in
// chunks. With `io` the grads come from host memory and the stepped params go
// back to it, on two copy streams: grads cross in the order the step consumes
// them (AdamW's, then each chunk's, largest chunk first), each group's compute
// starts when its copy lands, and each finished group's params start back at
// once, so the PCIe transfers in both directions overlap the compute.
static int enqueue_step(mmn_optim_t* h, float divisor, const HostIO* io) {
  NvtxRange range_step(io ? "mmn.step_host" : "mmn.step");
  cudaStream_t s = h->work;
  const bool tm = h->timing && !io;
  cudaEvent_t* ev = nullptr;
  if (tm) {
    const size_t k = h->ev_used % mmn_optim::kTimedSteps;
    if (k == h->ev_sets.size()) {
      std::array<cudaEvent_t, 9> set{};
      for (auto& e : set) MMN_CUDA_TRY(cudaEventCreate(&e));
      h->ev_sets.push_back(set);
    }
    ev = h->ev_sets[k].data();
    ++h->ev_used;
  }
  const bool bf = h->cfg.grad_dtype == MMN_DTYPE_BF16;
  const int R = h->cfg.rank;
  if (tm) MMN_CUDA_TRY(cudaEventRecord(ev[0], s));

  // ---- grads in (host steps), job by job
  if (io) {
    MMN_CUDA_TRY(cudaStreamWaitEvent(h->h2d, h->in_ev, 0));
    for (size_t j = 0; j < h->jobs.size(); ++j) {
      const int job = h->jobs[j];
      if (job >= 0) {
        for (int i : h->chunk_slots[job]) MMN_TRY_RC(grad_in(h, io, i, 0, h->slots[i].numel));
      } else {
        for (const auto& pc : h->apart_pieces[-1 - job]) MMN_TRY_RC(grad_in(h, io, pc.slot, pc.lo, pc.hi));
      }
      MMN_CUDA_TRY(cudaEventRecord(h->h2d_ev[j], h->h2d));
    }
    if (h->cfg.loss_scaling && h->cfg.world_size > 1 && !h->cfg.scan_shard) {
      // the non-finite scan reads every grad: the peers' parts come in too
      int64_t lo, hi;
      for (size_t i = 0; i < h->slots.size(); ++i) {
        stepped_range(h, h->slots[i], &lo, &hi);
        MMN_TRY_RC(grad_in(h, io, (int)i, 0, lo));
        MMN_TRY_RC(grad_in(h, io, (int)i, hi, h->slots[i].numel));
      }
    }
    MMN_CUDA_TRY(cudaEventRecord(h->h2d_ev.back(), h->h2d));
  }

  if (h->cfg.loss_scaling && !h->cfg.reduce_grads && !h->cfg.scan_shard) {
    // Every rank scans every grad (grads are replicated), so all ranks reach
    // the same skip decision without a collective. (With reduce_grads the
    // reduction, with scan_shard mmn_optim_scan_grads, already set the flag on
    // every rank.)
    if (io) MMN_CUDA_TRY(cudaStreamWaitEvent(s, h->h2d_ev.back(), 0));
    MMN_CUDA_TRY(cudaMemsetAsync(h->d_skip, 0, sizeof(int), s));
    const int64_t a_n = h->a_used4 * 4;
    if (bf) {
      launch_nonfinite_scan(nullptr, 0, static_cast<const __nv_bfloat16*>(h->ag), a_n, h->d_skip,
                            h->ctx.num_sms, s);
      launch_nonfinite_scan(nullptr, 0, static_cast<const __nv_bfloat16*>(h->mg), h->m_total,
                            h->d_skip, h->ctx.num_sms, s);
    } else {
      launch_nonfinite_scan(static_cast<const float*>(h->ag), a_n, nullptr, 0, h->d_skip,
                            h->ctx.num_sms, s);
      launch_nonfinite_scan(static_cast<const float*>(h->mg), h->m_total, nullptr, 0, h->d_skip,
                            h->ctx.num_sms, s);
    }
  }
  const int* skip = h->cfg.loss_scaling ? h->d_skip : nullptr;
  const float* gscale = h->cfg.loss_scaling ? h->d_scale : nullptr;

  // ---- AdamW on the side stream: one launch over this rank's range, or (host
  // steps) one per part, each after its grads landed
  {
    NvtxRange range_adamw("mmn.adamw");
    MMN_CUDA_TRY(cudaEventRecord(h->fork, s));
    MMN_CUDA_TRY(cudaStreamWaitEvent(h->side, h->fork, 0));
    if (tm) MMN_CUDA_TRY(cudaEventRecord(ev[1], h->side));
    AdamwArgs a{};
    a.p = h->ap;
    a.g = bf ? nullptr : static_cast<const float*>(h->ag);
    a.g_bf16 = bf ? static_cast<const __nv_bfloat16*>(h->ag) : nullptr;
    a.m = h->am;
    a.v = h->av;
    a.p_bf16 = h->ap16;
    a.segs = h->d_segs;
    a.chunk_seg = h->d_chunk_seg;
    a.bc_table = h->bc.dev;
    a.t_sat = h->bc.t_sat;
    a.step_base = h->d_step;
    a.skip = skip;
    a.grad_scale = gscale;
    a.lr = h->cfg.adamw.lr;
    a.b1 = h->cfg.adamw.beta1;
    a.b2 = h->cfg.adamw.beta2;
    a.eps = h->cfg.adamw.eps;
    a.wd = h->cfg.adamw.weight_decay;
    a.grad_divisor = divisor;
    a.fresh_state = h->cfg.fresh_state;
    void* a_src = h->cfg.bf16_param_shadow ? (void*)h->ap16 : (void*)h->ap;
    if (io) {
      for (size_t j = 0; j < h->jobs.size(); ++j) {
        if (h->jobs[j] >= 0) continue;
        const int p = -1 - h->jobs[j];
        MMN_CUDA_TRY(cudaStreamWaitEvent(h->side, h->h2d_ev[j], 0));
        a.begin4 = h->apart_begin4[p];
        a.end4 = h->apart_end4[p];
        launch_adamw(a, h->ctx.num_sms, h->side);
        MMN_CUDA_TRY(cudaGetLastError());
        MMN_CUDA_TRY(cudaEventRecord(h->apart_ev[p], h->side));
        if (h->n_peers)
          MMN_TRY_RC(copy_to_peers(h, h->apart_ev[p], a_src, h->peer_a, a.begin4 * 4, a.end4 * 4));
      }
    } else {
      a.begin4 = std::min<long long>(h->a_region4 * R, h->a_used4);
      a.end4 = std::min<long long>(h->a_region4 * (R + 1), h->a_used4);
      launch_adamw(a, h->ctx.num_sms, h->side);
      MMN_CUDA_TRY(cudaGetLastError());
      if (h->n_peers) {
        // this rank's AdamW range goes to every peer while the Muon work runs
        MMN_CUDA_TRY(cudaEventRecord(h->adamw_ev, h->side));
        MMN_TRY_RC(copy_to_peers(h, h->adamw_ev, a_src, h->peer_a, a.begin4 * 4, a.end4 * 4));
      }
    }
    if (tm) MMN_CUDA_TRY(cudaEventRecord(ev[2], h->side));
    MMN_CUDA_TRY(cudaEventRecord(h->join, h->side));
  }

  // ---- Muon on the work stream, chunk by chunk
  if (tm) MMN_CUDA_TRY(cudaEventRecord(ev[3], s));
  if (!h->mats.empty()) {
    MuonArgs m{};
    m.p = h->mp;
    m.g = bf ? nullptr : static_cast<const float*>(h->mg);
    m.g_bf16 = bf ? static_cast<const __nv_bfloat16*>(h->mg) : nullptr;
    m.vel = h->mvel;
    m.p_bf16 = h->mp16;
    m.cls = h->d_cls_in;
    m.partials = h->d_partials;
    m.norms = h->d_norms;
    m.skip = skip;
    m.grad_scale = gscale;
    m.momentum = h->cfg.muon.momentum;
    m.nesterov = h->cfg.muon.nesterov;
    m.grad_divisor = divisor;
    m.fresh_state = h->cfg.fresh_state;
    m.apply_divides_norm = h->cfg.muon.ns_steps == 0;
    m.vec_ok = 1;  // arena bases come from cudaMalloc; offsets are 64-element aligned
    m.x_mode = h->cfg.ns_mode == MMN_NS_FP32 ? 2 : (h->cfg.ns_mode == MMN_NS_TF32 ? 1 : 0);
    m.norm_scalar_rows = h->norm_scalar_rows;
    auto select = [&](size_t k) {
      m.mats = h->d_mats + h->chunk_mat0[k];
      m.nmat = h->chunk_mat0[k + 1] - h->chunk_mat0[k];
      m.tile_begin = h->chunk_tile0[k];
      m.total_tiles = h->chunk_tile0[k + 1] - h->chunk_tile0[k];
    };
    // momentum and bf16 cast of chunk k, and its norms unless they come later
    // for every chunk at once
    auto prologue = [&](size_t k, bool norms) -> int {
      NvtxRange r("mmn.muon_momentum");
      select(k);
      m.cls = h->d_cls_in;
      launch_muon_momentum(m, h->ctx.num_sms, s);
      if (norms) launch_muon_norms(m, s, h->chunk_norm_cluster[k]);
      MMN_CUDA_TRY(cudaGetLastError());
      return MMN_OK;
    };
    // The last Newton-Schulz iteration applies p -= lr*scale*O itself
    // (lib.rs:169-174); with zero iterations the update kernel does it.
    const bool fuse = h->cfg.muon.ns_steps >= 1;
    auto newton_schulz = [&](size_t k) -> int {
      NvtxRange r("mmn.newton_schulz");
      NsFused f;
      f.p = h->mp;
      f.p_bf16 = h->mp16;
      f.apply = h->d_apply + h->cls_base[k];
      std::string err;
      if (ns_class_run(h->classes[k], h->cfg.muon.ns_steps, h->cfg.ns_mode, h->ctx.status,
                       h->ctx.num_sms, s, &err, fuse ? &f : nullptr, skip) < 0)
        return fail(MMN_E_CUDA, err);
      if (!fuse) {
        select(k);
        m.cls = h->d_cls_out;
        launch_muon_apply(m, h->ctx.num_sms, s);
        MMN_CUDA_TRY(cudaGetLastError());
      }
      if (h->n_peers || io) MMN_CUDA_TRY(cudaEventRecord(h->chunk_ev[k], s));
      if (h->n_peers) {
        // the chunk's parameters are final: copy engines push them over NVLink
        // while the next chunk computes
        MMN_TRY_RC(copy_to_peers(h, h->chunk_ev[k],
                                 h->cfg.bf16_param_shadow ? (void*)h->mp16 : (void*)h->mp,
                                 h->peer_m, h->chunk_begin[k], h->chunk_end[k]));
      }
      return MMN_OK;
    };
    if (io) {
      for (size_t j = 0; j < h->jobs.size(); ++j) {
        if (h->jobs[j] < 0) continue;
        MMN_CUDA_TRY(cudaStreamWaitEvent(s, h->h2d_ev[j], 0));
        MMN_TRY_RC(prologue(h->jobs[j], true));
        MMN_TRY_RC(newton_schulz(h->jobs[j]));
      }
    } else {
      for (int k : h->jobs)
        if (k >= 0) MMN_TRY_RC(prologue(k, false));
      if (tm) MMN_CUDA_TRY(cudaEventRecord(ev[8], s));
      // the norms of every matrix in one launch: one CTA per matrix, largest
      // first, so the long sequential sums of the large matrices run side by side
      m.mats = h->d_mats;
      m.nmat = (int)h->mats.size();
      m.tile_begin = 0;
      m.total_tiles = h->total_tiles;
      m.cls = h->d_cls_in;
      launch_muon_norms(m, s, h->norm_cluster);
      MMN_CUDA_TRY(cudaGetLastError());
      if (tm) MMN_CUDA_TRY(cudaEventRecord(ev[4], s));
      for (int k : h->jobs)
        if (k >= 0) MMN_TRY_RC(newton_schulz(k));
    }
    if (tm) MMN_CUDA_TRY(cudaEventRecord(ev[5], s));
  } else if (tm) {
    MMN_CUDA_TRY(cudaEventRecord(ev[8], s));
    MMN_CUDA_TRY(cudaEventRecord(ev[4], s));
    MMN_CUDA_TRY(cudaEventRecord(ev[5], s));
  }
  if (tm) MMN_CUDA_TRY(cudaEventRecord(ev[6], s));

  // ---- params out (host steps), job by job, queued after all compute so that
  // a copy into pageable memory, which blocks the host, cannot hold back a launch
  if (io) {
    for (int job : h->jobs) {
      if (job >= 0) {
        MMN_CUDA_TRY(cudaStreamWaitEvent(h->d2h, h->chunk_ev[job], 0));
        for (int i : h->chunk_slots[job]) MMN_TRY_RC(param_out(h, io, i, 0, h->slots[i].numel));
      } else {
        MMN_CUDA_TRY(cudaStreamWaitEvent(h->d2h, h->apart_ev[-1 - job], 0));
        for (const auto& pc : h->apart_pieces[-1 - job]) MMN_TRY_RC(param_out(h, io, pc.slot, pc.lo, pc.hi));
      }
    }
    MMN_CUDA_TRY(cudaEventRecord(h->d2h_done, h->d2h));
    MMN_CUDA_TRY(cudaStreamWaitEvent(s, h->d2h_done, 0));
  }
  MMN_CUDA_TRY(cudaStreamWaitEvent(s, h->join, 0));
  for (int r = 0; r < h->n_peers; ++r) {
    MMN_CUDA_TRY(cudaEventRecord(h->xfer_done[r], h->xfer[r]));
    MMN_CUDA_TRY(cudaStreamWaitEvent(s, h->xfer_done[r], 0));
  }
  StepTail t{};
  t.step_counter = h->d_step;
  t.adamw_calls = h->n_adamw;
  t.skip = h->cfg.loss_scaling ? h->d_skip : nullptr;
  t.reset_skip = h->cfg.reduce_grads || h->cfg.scan_shard;
  t.grad_scale = h->cfg.loss_scaling ? h->d_scale : nullptr;
  t.good_steps = h->d_good;
  t.growth_interval = h->cfg.growth_interval > 0 ? h->cfg.growth_interval : 2000;
  t.skipped_total = h->d_skipped;
  launch_step_tail(t, s);
  MMN_CUDA_TRY(cudaGetLastError());
  if (tm) MMN_CUDA_TRY(cudaEventRecord(ev[7], s));
  return MMN_OK;
}

// reduce_grads and scan_shard handles step only grads that went through
// mmn_optim_reduce_grads / mmn_optim_scan_grads since the last step: without
// it the step would use this rank's unreduced grads, or no rank's non-finite
// verdict.
static int take_grads(mmn_optim_t* h) {
  if (!h->cfg.reduce_grads && !h->cfg.scan_shard) return MMN_OK;
  if (!h->grads_ready)
    return fail(MMN_E_STATE, h->cfg.reduce_grads ? "call mmn_optim_reduce_grads before each step"
                                                 : "call mmn_optim_scan_grads before each step");
  h->grads_ready = false;
  return MMN_OK;
}

extern "C" int mmn_optim_step(mmn_optim_t* h, float grad_divisor) {
  if (!h) return fail(MMN_E_INVALID, "null handle");
  if (!h->finalized) return fail(MMN_E_STATE, "finalize before step");
  if (!(grad_divisor > 0.0f)) return fail(MMN_E_INVALID, "grad_divisor must be > 0");
  MMN_TRY_RC(take_grads(h));
  DeviceGuard g(h->ctx.device);
  // The step runs on the handle's own work stream, ordered after everything
  // already queued on the caller's stream and before anything queued there
  // later. Capture therefore never touches the caller's stream (which may be
  // the legacy default stream, where capture is not allowed).
  MMN_CUDA_TRY(cudaEventRecord(h->in_ev, h->ctx.stream));
  MMN_CUDA_TRY(cudaStreamWaitEvent(h->work, h->in_ev, 0));
  int rc = MMN_OK;
  if (!h->cfg.use_graph || h->timing) {
    rc = enqueue_step(h, grad_divisor, nullptr);
  } else {
    if (h->graph && h->graph_divisor != grad_divisor) {
      cudaGraphExecDestroy(h->graph);
      h->graph = nullptr;
    }
    if (!h->graph) {
      cudaGraph_t graph = nullptr;
      MMN_CUDA_TRY(cudaStreamBeginCapture(h->work, cudaStreamCaptureModeThreadLocal));
      rc = enqueue_step(h, grad_divisor, nullptr);
      cudaError_t e = cudaStreamEndCapture(h->work, &graph);
      if (rc != MMN_OK) {
        if (graph) cudaGraphDestroy(graph);
        return rc;
      }
      if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
      e = cudaGraphInstantiate(&h->graph, graph, 0);
      cudaGraphDestroy(graph);
      if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
      h->graph_divisor = grad_divisor;
    }
    MMN_CUDA_TRY(cudaGraphLaunch(h->graph, h->work));
  }
  MMN_CUDA_TRY(cudaEventRecord(h->out_ev, h->work));
  MMN_CUDA_TRY(cudaStreamWaitEvent(h->ctx.stream, h->out_ev, 0));
  return rc;
}

extern "C" int mmn_optim_step_host(mmn_optim_t* h, const void* const* grads,
                                   float* const* params, float grad_divisor) {
  if (!h) return fail(MMN_E_INVALID, "null handle");
  if (!h->finalized) return fail(MMN_E_STATE, "finalize before step");
  if (!grads || !params) return fail(MMN_E_INVALID, "grads and params must be slot arrays");
  if (!(grad_divisor > 0.0f)) return fail(MMN_E_INVALID, "grad_divisor must be > 0");
  if (h->cfg.reduce_grads)
    return fail(MMN_E_UNSUPPORTED, "a step from host memory takes already-reduced grads");
  if (h->cfg.scan_shard)
    for (size_t i = 0; i < h->slots.size(); ++i)
      if (grads[i])
        return fail(MMN_E_STATE,
                    "with scan_shard the grads go in through mmn_optim_scan_grads, before "
                    "the step: pass null grads here");
  MMN_TRY_RC(take_grads(h));
  DeviceGuard g(h->ctx.device);
  MMN_CUDA_TRY(cudaEventRecord(h->in_ev, h->ctx.stream));
  MMN_CUDA_TRY(cudaStreamWaitEvent(h->work, h->in_ev, 0));
  HostIO io{grads, params};
  const int rc = enqueue_step(h, grad_divisor, &io);
  // join the copy streams back even after an enqueue error, so that nothing
  // still in flight outlives the call unordered
  MMN_CUDA_TRY(cudaEventRecord(h->out_ev, h->h2d));
  MMN_CUDA_TRY(cudaStreamWaitEvent(h->work, h->out_ev, 0));
  MMN_CUDA_TRY(cudaEventRecord(h->out_ev, h->d2h));
  MMN_CUDA_TRY(cudaStreamWaitEvent(h->work, h->out_ev, 0));
  MMN_CUDA_TRY(cudaEventRecord(h->out_ev, h->work));
  MMN_CUDA_TRY(cudaStreamWaitEvent(h->ctx.stream, h->out_ev, 0));
  if (rc != MMN_OK) return rc;
  MMN_CUDA_TRY(cudaEventSynchronize(h->out_ev));
  return h->ctx.check_status();
}

extern "C" int mmn_optim_sync(mmn_optim_t* h) {
  if (!h) return fail(MMN_E_INVALID, "null handle");
  DeviceGuard g(h->ctx.device);
  return h->ctx.check_status();
}

extern "C" int mmn_optim_loss_scale(mmn_optim_t* h, float* scale, int64_t* skipped_steps) {
  if (!h || !h->finalized) return fail(MMN_E_STATE, "finalize first");
  DeviceGuard g(h->ctx.device);
  MMN_CUDA_TRY(cudaStreamSynchronize(h->ctx.stream));
  float sc = 0.0f;
  int sk = 0;
  MMN_CUDA_TRY(cudaMemcpy(&sc, h->d_scale, sizeof(float), cudaMemcpyDeviceToHost));
  MMN_CUDA_TRY(cudaMemcpy(&sk, h->d_skipped, sizeof(int), cudaMemcpyDeviceToHost));
  if (scale) *scale = sc;
  if (skipped_steps) *skipped_steps = sk;
  return MMN_OK;
}

extern "C" int mmn_optim_get_loss_state(mmn_optim_t* h, float* scale, int64_t* skipped_steps,
                                        int32_t* good_steps) {
  if (!h || !h->finalized) return fail(MMN_E_STATE, "finalize first");
  DeviceGuard g(h->ctx.device);
  MMN_CUDA_TRY(cudaStreamSynchronize(h->ctx.stream));
  float sc = 0.0f;
  int sk = 0, gd = 0;
  MMN_CUDA_TRY(cudaMemcpy(&sc, h->d_scale, sizeof(float), cudaMemcpyDeviceToHost));
  MMN_CUDA_TRY(cudaMemcpy(&sk, h->d_skipped, sizeof(int), cudaMemcpyDeviceToHost));
  MMN_CUDA_TRY(cudaMemcpy(&gd, h->d_good, sizeof(int), cudaMemcpyDeviceToHost));
  if (scale) *scale = sc;
  if (skipped_steps) *skipped_steps = sk;
  if (good_steps) *good_steps = gd;
  return MMN_OK;
}

extern "C" int mmn_optim_set_loss_state(mmn_optim_t* h, float scale, int64_t skipped_steps,
                                        int32_t good_steps) {
  if (!h || !h->finalized) return fail(MMN_E_STATE, "finalize first");
  if (!(scale > 0.0f) || skipped_steps < 0 || skipped_steps > INT32_MAX || good_steps < 0)
    return fail(MMN_E_INVALID, "bad loss-scaling state");
  DeviceGuard g(h->ctx.device);
  const int sk = (int)skipped_steps, gd = good_steps;
  MMN_CUDA_TRY(cudaMemcpyAsync(h->d_scale, &scale, sizeof(float), cudaMemcpyHostToDevice,
                               h->ctx.stream));
  MMN_CUDA_TRY(cudaMemcpyAsync(h->d_skipped, &sk, sizeof(int), cudaMemcpyHostToDevice,
                               h->ctx.stream));
  MMN_CUDA_TRY(cudaMemcpyAsync(h->d_good, &gd, sizeof(int), cudaMemcpyHostToDevice,
                               h->ctx.stream));
  MMN_CUDA_TRY(cudaStreamSynchronize(h->ctx.stream));
  return MMN_OK;
}

extern "C" int mmn_optim_slot_owner(mmn_optim_t* h, int slot, int* owner_rank) {
  int rc = check_slot(h, slot);
  if (rc != MMN_OK) return rc;
  if (owner_rank) *owner_rank = h->slots[slot].route == MMN_ROUTE_MUON ? h->slots[slot].owner : -1;
  return MMN_OK;
}

extern "C" int mmn_optim_get_gather_layout(mmn_optim_t* h, mmn_optim_gather_layout* out) {
  if (!h || !out) return fail(MMN_E_INVALID, "null argument");
  if (!h->finalized) return fail(MMN_E_STATE, "finalize first");
  out->adamw_param = h->ap;
  out->adamw_param_bf16 = h->ap16;
  out->adamw_region = h->a_region4 * 4;
  out->muon_param = h->mp;
  out->muon_param_bf16 = h->mp16;
  out->muon_region = h->m_region;
  return MMN_OK;
}

namespace {
// What one rank publishes for the fused exchange.
struct IpcBlob {
  uint32_t magic;
  int32_t rank, world;
  int32_t shadow;
  int64_t a_total4, m_total;
  int32_t grad_dtype, reduce_grads, scan_shard;
  cudaIpcMemHandle_t ap, mp, ap16, mp16;
  cudaIpcMemHandle_t ga, gm;  // grad arenas (reduce_grads)
  cudaIpcMemHandle_t skip;    // skip flag (reduce_grads or scan_shard)
};
static_assert(sizeof(IpcBlob) <= MMN_IPC_BLOB_BYTES, "IPC blob size");
constexpr uint32_t kIpcMagic = 0x4D4D4E31u;  // "MMN1"
}  // namespace

extern "C" int mmn_optim_export_ipc(mmn_optim_t* h, void* blob) {
  if (!h || !blob) return fail(MMN_E_INVALID, "null argument");
  if (!h->finalized) return fail(MMN_E_STATE, "finalize first");
  DeviceGuard g(h->ctx.device);
  IpcBlob b;
  memset(&b, 0, sizeof(b));
  b.magic = kIpcMagic;
  b.rank = h->cfg.rank;
  b.world = h->cfg.world_size;
  b.shadow = h->cfg.bf16_param_shadow;
  b.a_total4 = h->a_total4;
  b.m_total = h->m_total;
  b.grad_dtype = h->cfg.grad_dtype;
  b.reduce_grads = h->cfg.reduce_grads;
  b.scan_shard = h->cfg.scan_shard;
  MMN_CUDA_TRY(cudaIpcGetMemHandle(&b.ap, h->ap));
  MMN_CUDA_TRY(cudaIpcGetMemHandle(&b.mp, h->mp));
  if (b.shadow) {
    MMN_CUDA_TRY(cudaIpcGetMemHandle(&b.ap16, h->ap16));
    MMN_CUDA_TRY(cudaIpcGetMemHandle(&b.mp16, h->mp16));
  }
  if (b.reduce_grads) {
    MMN_CUDA_TRY(cudaIpcGetMemHandle(&b.ga, h->ag));
    MMN_CUDA_TRY(cudaIpcGetMemHandle(&b.gm, h->mg));
  }
  if (b.reduce_grads || b.scan_shard) MMN_CUDA_TRY(cudaIpcGetMemHandle(&b.skip, h->d_skip));
  memset(blob, 0, MMN_IPC_BLOB_BYTES);
  memcpy(blob, &b, sizeof(b));
  return MMN_OK;
}

extern "C" int mmn_optim_connect_peers(mmn_optim_t* h, const void* blobs) {
  if (!h || !blobs) return fail(MMN_E_INVALID, "null argument");
  if (!h->finalized) return fail(MMN_E_STATE, "finalize first");
  const int W = h->cfg.world_size, R = h->cfg.rank;
  constexpr int kMaxPeers = 7;
  if (W - 1 > kMaxPeers) return fail(MMN_E_UNSUPPORTED, "at most 8 ranks share the exchange");
  if (!h->peer_maps.empty()) return fail(MMN_E_STATE, "peers already connected");
  DeviceGuard g(h->ctx.device);
  const uint8_t* raw = static_cast<const uint8_t*>(blobs);
  int n_peers = 0;
  void* peer_a[8] = {};
  void* peer_m[8] = {};
  const void* rank_ga[8] = {};
  const void* rank_gm[8] = {};
  int* rank_skip[8] = {};
  std::vector<void*> maps;
  auto open = [&](const cudaIpcMemHandle_t& hd, void** out) -> int {
    cudaError_t e = cudaIpcOpenMemHandle(out, hd, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    maps.push_back(*out);
    return MMN_OK;
  };
  int rc = MMN_OK;
  for (int r = 0; r < W && rc == MMN_OK; ++r) {
    IpcBlob b;
    memcpy(&b, raw + (size_t)r * MMN_IPC_BLOB_BYTES, sizeof(b));
    if (b.magic != kIpcMagic || b.rank != r || b.world != W ||
        b.shadow != h->cfg.bf16_param_shadow || b.a_total4 != h->a_total4 ||
        b.m_total != h->m_total || b.grad_dtype != h->cfg.grad_dtype ||
        b.reduce_grads != h->cfg.reduce_grads || b.scan_shard != h->cfg.scan_shard) {
      rc = fail(MMN_E_INVALID, "peer blob does not match this rank's layout");
      break;
    }
    if (r == R) {
      rank_ga[r] = h->ag;
      rank_gm[r] = h->mg;
      rank_skip[r] = h->d_skip;
      continue;
    }
    void *ap = nullptr, *mp = nullptr;
    const bool sh = h->cfg.bf16_param_shadow;
    if ((rc = open(sh ? b.ap16 : b.ap, &ap)) != MMN_OK || (rc = open(sh ? b.mp16 : b.mp, &mp)) != MMN_OK)
      break;
    peer_a[n_peers] = ap;
    peer_m[n_peers] = mp;
    ++n_peers;
    if (h->cfg.reduce_grads) {
      void *ga = nullptr, *gm = nullptr;
      if ((rc = open(b.ga, &ga)) != MMN_OK || (rc = open(b.gm, &gm)) != MMN_OK) break;
      rank_ga[r] = ga;
      rank_gm[r] = gm;
    }
    if (h->cfg.reduce_grads || h->cfg.scan_shard) {
      void* sk = nullptr;
      if ((rc = open(b.skip, &sk)) != MMN_OK) break;
      rank_skip[r] = static_cast<int*>(sk);
    }
  }
  auto undo = [&](int code) {
    for (void* p : maps) cudaIpcCloseMemHandle(p);
    return code;
  };
  if (rc != MMN_OK) return undo(rc);
  h->peer_maps = maps;
  h->n_peers = n_peers;
  for (int k = 0; k < n_peers; ++k) {
    h->peer_a[k] = peer_a[k];
    h->peer_m[k] = peer_m[k];
  }
  for (int r = 0; r < W; ++r) {
    h->rank_ga[r] = rank_ga[r];
    h->rank_gm[r] = rank_gm[r];
    h->rank_skip[r] = rank_skip[r];
  }
  h->reduce_ready = h->cfg.reduce_grads != 0 || h->cfg.scan_shard != 0;
  if (h->graph) {  // the captured step must be re-captured with the peers
    cudaGraphExecDestroy(h->graph);
    h->graph = nullptr;
  }
  return MMN_OK;
}

extern "C" int mmn_optim_reduce_grads(mmn_optim_t* h) {
  NvtxRange range("mmn.reduce_grads");
  if (!h) return fail(MMN_E_INVALID, "null handle");
  if (!h->finalized) return fail(MMN_E_STATE, "finalize first");
  if (!h->cfg.reduce_grads || h->cfg.world_size < 2)
    return fail(MMN_E_STATE, "create the handle with reduce_grads = 1 and world_size > 1");
  if (!h->reduce_ready) return fail(MMN_E_STATE, "connect the peers first");
  DeviceGuard g(h->ctx.device);
  const int W = h->cfg.world_size, R = h->cfg.rank;
  MMN_CUDA_TRY(cudaEventRecord(h->in_ev, h->ctx.stream));
  MMN_CUDA_TRY(cudaStreamWaitEvent(h->work, h->in_ev, 0));
  GradReduceArgs a{};
  a.world = W;
  a.bf16 = h->cfg.grad_dtype == MMN_DTYPE_BF16;
  a.scan = h->cfg.loss_scaling;
  for (int r = 0; r < W; ++r) a.skip_flags[r] = h->rank_skip[r];
  // this rank's AdamW range
  for (int r = 0; r < W; ++r) a.src[r] = h->rank_ga[r];
  a.dst = h->ag;
  a.begin = std::min<int64_t>(h->a_region4 * R, h->a_used4) * 4;
  a.end = std::min<int64_t>(h->a_region4 * (R + 1), h->a_used4) * 4;
  launch_grad_reduce(a, h->ctx.num_sms, h->work);
  MMN_CUDA_TRY(cudaGetLastError());
  // this rank's Muon matrices
  for (int r = 0; r < W; ++r) a.src[r] = h->rank_gm[r];
  a.dst = h->mg;
  a.begin = h->m_own_begin;
  a.end = h->m_own_end;
  launch_grad_reduce(a, h->ctx.num_sms, h->work);
  MMN_CUDA_TRY(cudaGetLastError());
  MMN_CUDA_TRY(cudaEventRecord(h->out_ev, h->work));
  MMN_CUDA_TRY(cudaStreamWaitEvent(h->ctx.stream, h->out_ev, 0));
  h->grads_ready = true;
  return MMN_OK;
}

extern "C" int mmn_optim_scan_grads(mmn_optim_t* h, const void* const* grads) {
  NvtxRange range("mmn.scan_grads");
  if (!h) return fail(MMN_E_INVALID, "null handle");
  if (!h->finalized) return fail(MMN_E_STATE, "finalize first");
  if (!h->cfg.scan_shard) return fail(MMN_E_STATE, "create the handle with scan_shard = 1");
  if (!h->reduce_ready) return fail(MMN_E_STATE, "connect the peers first");
  DeviceGuard g(h->ctx.device);
  const int W = h->cfg.world_size, R = h->cfg.rank;
  cudaStream_t s = h->ctx.stream;
  if (grads) {
    // this rank's parts of the host grads in first, on the copy stream
    HostIO io{grads, nullptr};
    MMN_CUDA_TRY(cudaEventRecord(h->in_ev, s));
    MMN_CUDA_TRY(cudaStreamWaitEvent(h->h2d, h->in_ev, 0));
    int64_t lo, hi;
    for (size_t i = 0; i < h->slots.size(); ++i)
      if (stepped_range(h, h->slots[i], &lo, &hi)) MMN_TRY_RC(grad_in(h, &io, (int)i, lo, hi));
    MMN_CUDA_TRY(cudaEventRecord(h->out_ev, h->h2d));
    MMN_CUDA_TRY(cudaStreamWaitEvent(s, h->out_ev, 0));
  }
  RankFlags f{};
  f.n = W;
  for (int r = 0; r < W; ++r) f.flag[r] = h->rank_skip[r];
  const bool bf = h->cfg.grad_dtype == MMN_DTYPE_BF16;
  const size_t gsz = bf ? 2 : 4;
  const int64_t alo = std::min<int64_t>(h->a_region4 * R, h->a_used4) * 4;
  const int64_t ahi = std::min<int64_t>(h->a_region4 * (R + 1), h->a_used4) * 4;
  const uint8_t* ag = static_cast<const uint8_t*>(h->ag) + (size_t)alo * gsz;
  const uint8_t* mg = static_cast<const uint8_t*>(h->mg) + (size_t)h->m_own_begin * gsz;
  const int64_t an = ahi - alo, mn = h->m_own_end - h->m_own_begin;
  if (bf) {
    launch_nonfinite_scan_ranks(nullptr, 0, reinterpret_cast<const __nv_bfloat16*>(ag), an, f,
                                h->ctx.num_sms, s);
    launch_nonfinite_scan_ranks(nullptr, 0, reinterpret_cast<const __nv_bfloat16*>(mg), mn, f,
                                h->ctx.num_sms, s);
  } else {
    launch_nonfinite_scan_ranks(reinterpret_cast<const float*>(ag), an, nullptr, 0, f,
                                h->ctx.num_sms, s);
    launch_nonfinite_scan_ranks(reinterpret_cast<const float*>(mg), mn, nullptr, 0, f,
                                h->ctx.num_sms, s);
  }
  MMN_CUDA_TRY(cudaGetLastError());
  if (grads) MMN_CUDA_TRY(cudaStreamSynchronize(s));  // the host buffers may be reused
  h->grads_ready = true;
  return MMN_OK;
}

extern "C" int mmn_optim_param_counts(mmn_optim_t* h, int64_t* total, int64_t* adamw,
                                      int64_t* muon) {
  if (!h || !h->finalized) return fail(MMN_E_STATE, "finalize first");
  if (total) *total = h->n_params;
  if (adamw) *adamw = h->n_adamw_params;
  if (muon) *muon = h->n_muon_params;
  return MMN_OK;
}

extern "C" int mmn_optim_ns_flops(mmn_optim_t* h, double* flops) {
  if (!h || !h->finalized || !flops) return fail(MMN_E_STATE, "finalize first");
  *flops = h->ns_flops;
  return MMN_OK;
}

extern "C" int mmn_optim_kernel_launches(mmn_optim_t* h, int64_t* per_step,
                                         int64_t* per_reduce) {
  if (!h || !h->finalized) return fail(MMN_E_STATE, "finalize first");
  const int R = h->cfg.rank;
  const bool adamw = std::min<int64_t>(h->a_region4 * (R + 1), h->a_used4) >
                     std::min<int64_t>(h->a_region4 * R, h->a_used4);
  const int steps = h->cfg.muon.ns_steps;
  int64_t n = (adamw ? 1 : 0) + 1;  // AdamW, step tail
  if (h->cfg.loss_scaling && !h->cfg.reduce_grads && !h->cfg.scan_shard)
    n += 2;  // non-finite scans
  // per chunk: momentum, 3 GEMMs per iteration (or the update kernel); the
  // norms of every chunk in one launch (mmn_optim_step_host: one per chunk)
  const int64_t chunks = (int64_t)h->chunk_begin.size();
  n += chunks * (1 + (steps >= 1 ? 3 * steps : 1)) + (chunks ? 1 : 0);
  if (per_step) *per_step = n;
  // mmn_optim_reduce_grads, or mmn_optim_scan_grads: one launch per arena
  if (per_reduce) *per_reduce = (h->cfg.reduce_grads || h->cfg.scan_shard) ? 2 : 0;
  return MMN_OK;
}

extern "C" int mmn_optim_enable_timing(mmn_optim_t* h, int enable) {
  if (!h) return fail(MMN_E_INVALID, "null handle");
  h->timing = enable != 0;
  if (h->timing) h->ev_used = 0;  // a new averaging window
  return MMN_OK;
}

// Averages event intervals over the timed steps: out[i] = mean of
// ev[to[i]] - ev[from[i]].
static int phase_means(mmn_optim_t* h, const int* from, const int* to, int n_out, float* out) {
  if (!h->timing || h->ev_used == 0) return fail(MMN_E_STATE, "enable timing before the steps");
  DeviceGuard g(h->ctx.device);
  MMN_CUDA_TRY(cudaStreamSynchronize(h->ctx.stream));
  const size_t n = std::min(h->ev_used, mmn_optim::kTimedSteps);
  double acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (size_t k = 0; k < n; ++k) {
    const cudaEvent_t* ev = h->ev_sets[k].data();
    for (int i = 0; i < n_out; ++i) {
      float ms = 0.0f;
      MMN_CUDA_TRY(cudaEventElapsedTime(&ms, ev[from[i]], ev[to[i]]));
      acc[i] += ms;
    }
  }
  for (int i = 0; i < n_out; ++i) out[i] = (float)(acc[i] / (double)n);
  return MMN_OK;
}

extern "C" int mmn_optim_last_timing(mmn_optim_t* h, float* ms5) {
  if (!h || !ms5) return fail(MMN_E_INVALID, "null argument");
  const int from[5] = {1, 3, 4, 5, 0}, to[5] = {2, 4, 5, 6, 7};
  return phase_means(h, from, to, 5, ms5);
}

extern "C" int mmn_optim_last_timing_ex(mmn_optim_t* h, float* ms6) {
  if (!h || !ms6) return fail(MMN_E_INVALID, "null argument");
  // AdamW, momentum, norms, Newton-Schulz, update, step
  const int from[6] = {1, 3, 8, 4, 5, 0}, to[6] = {2, 8, 4, 5, 6, 7};
  return phase_means(h, from, to, 6, ms6);
}
