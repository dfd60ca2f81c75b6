// Per-call C ABI: one entry point per method of the reference's Rust optimizer
// types (crates/mmn-optim/src/lib.rs). State is device-resident and keyed by
// the caller's id, exactly like the reference's HashMaps.
#include <cstring>
#include <map>
#include <unordered_map>
#include <utility>

#include "capi_internal.cuh"
#include "elementwise.cuh"
#include "ns_engine.cuh"

namespace mmn {

// Copies `n` floats between host or device `src` and device `dst` on `s`.
static cudaError_t copy_in(float* dst, const float* src, int64_t n, int mem, cudaStream_t s) {
  return cudaMemcpyAsync(dst, src, (size_t)n * 4,
                         mem == MMN_MEM_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice, s);
}
static cudaError_t copy_out(float* dst, const float* src, int64_t n, int mem, cudaStream_t s) {
  return cudaMemcpyAsync(dst, src, (size_t)n * 4,
                         mem == MMN_MEM_HOST ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice, s);
}

static bool same_shape(const std::vector<int64_t>& a, const int64_t* b, int nd) {
  if ((int)a.size() != nd) return false;
  for (int i = 0; i < nd; ++i)
    if (a[i] != b[i]) return false;
  return true;
}

}  // namespace mmn

using namespace mmn;

// ===================================================================== AdamW
struct mmn_adamw {
  Ctx ctx;
  mmn_adamw_config cfg;
  uint64_t step = 0;
  struct State {
    float* m = nullptr;
    float* v = nullptr;
    int64_t numel = 0;
    std::vector<int64_t> shape;
  };
  std::unordered_map<uint64_t, State> state;
  BiasTable bc;
  Scratch sp, sg;
};

static int adamw_state(mmn_adamw* h, uint64_t id, const int64_t* shape, int ndim, int64_t numel,
                       mmn_adamw::State** out) {
  auto it = h->state.find(id);
  if (it != h->state.end()) {
    if (!same_shape(it->second.shape, shape, ndim))
      return fail(MMN_E_SHAPE, "param shape differs from the state registered for this id");
    *out = &it->second;
    return MMN_OK;
  }
  mmn_adamw::State st;
  st.numel = numel;
  st.shape.assign(shape, shape + ndim);
  const size_t bytes = (size_t)((numel + 3) / 4) * 16;
  if (bytes) {
    cudaError_t e = cudaMalloc(&st.m, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&st.v, bytes);
    if (e == cudaSuccess) e = cudaMemsetAsync(st.m, 0, bytes, h->ctx.stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(st.v, 0, bytes, h->ctx.stream);
    if (e != cudaSuccess) {
      if (st.m) cudaFree(st.m);
      if (st.v) cudaFree(st.v);
      return cuda_fail(e, "AdamW state allocation");
    }
  }
  *out = &(h->state[id] = st);
  return MMN_OK;
}

extern "C" int mmn_adamw_create(const mmn_adamw_config* cfg, int device, void* stream,
                                mmn_adamw_t** out) {
  if (!out) return fail(MMN_E_INVALID, "out is null");
  *out = nullptr;
  auto* h = new mmn_adamw();
  h->cfg = cfg ? *cfg : mmn_adamw_config_default();
  int rc = h->ctx.init(device, stream);
  if (rc == MMN_OK) {
    DeviceGuard g(device);
    rc = h->bc.build(h->cfg.beta1, h->cfg.beta2);
  }
  if (rc != MMN_OK) {
    h->ctx.release();
    delete h;
    return rc;
  }
  *out = h;
  return MMN_OK;
}

extern "C" int mmn_adamw_destroy(mmn_adamw_t* h) {
  if (!h) return MMN_OK;
  DeviceGuard g(h->ctx.device);
  cudaStreamSynchronize(h->ctx.stream);
  for (auto& kv : h->state) {
    cudaFree(kv.second.m);
    cudaFree(kv.second.v);
  }
  h->bc.release();
  h->sp.release();
  h->sg.release();
  h->ctx.release();
  delete h;
  return MMN_OK;
}

extern "C" int mmn_adamw_step_param(mmn_adamw_t* h, uint64_t id, float* param, const float* grad,
                                    const int64_t* shape, int ndim, float grad_divisor, int mem) {
  if (!h || !param || !grad) return fail(MMN_E_INVALID, "null handle, param or grad");
  if (mem != MMN_MEM_HOST && mem != MMN_MEM_DEVICE) return fail(MMN_E_INVALID, "bad mem kind");
  if (!(grad_divisor > 0.0f)) return fail(MMN_E_INVALID, "grad_divisor must be > 0");
  int rc;
  const int64_t numel = shape_numel(shape, ndim, &rc);
  if (rc != MMN_OK) return rc;
  DeviceGuard g(h->ctx.device);
  if (mem == MMN_MEM_DEVICE && numel > 0) {
    if ((rc = check_device_ptr(param, h->ctx.device, "param")) != MMN_OK) return rc;
    if ((rc = check_device_ptr(grad, h->ctx.device, "grad")) != MMN_OK) return rc;
  }
  mmn_adamw::State* st = nullptr;
  if ((rc = adamw_state(h, id, shape, ndim, numel, &st)) != MMN_OK) return rc;
  h->step += 1;  // lib.rs:42, on every call
  if (numel == 0) return MMN_OK;
  const int64_t n4 = (numel + 3) / 4;
  cudaStream_t s = h->ctx.stream;
  const bool direct = mem == MMN_MEM_DEVICE && numel % 4 == 0 &&
                      (reinterpret_cast<uintptr_t>(param) % 16) == 0 &&
                      (reinterpret_cast<uintptr_t>(grad) % 16) == 0;
  float* p = param;
  const float* gp = grad;
  if (!direct) {
    if ((rc = h->sp.ensure((size_t)n4 * 16)) != MMN_OK) return rc;
    if ((rc = h->sg.ensure((size_t)n4 * 16)) != MMN_OK) return rc;
    p = static_cast<float*>(h->sp.ptr);
    float* gs = static_cast<float*>(h->sg.ptr);
    MMN_CUDA_TRY(cudaMemsetAsync(p + (n4 - 1) * 4, 0, 16, s));
    MMN_CUDA_TRY(cudaMemsetAsync(gs + (n4 - 1) * 4, 0, 16, s));
    MMN_CUDA_TRY(copy_in(p, param, numel, mem, s));
    MMN_CUDA_TRY(copy_in(gs, grad, numel, mem, s));
    gp = gs;
  }
  AdamwArgs a{};
  a.p = p;
  a.g = gp;
  a.m = st->m;
  a.v = st->v;
  a.segs = nullptr;
  a.seg0.start4 = 0;
  a.seg0.end4 = n4;
  a.seg0.t_offset = 0;
  a.begin4 = 0;
  a.end4 = n4;
  a.bc_table = h->bc.dev;
  a.t_sat = h->bc.t_sat;
  a.step_base = nullptr;
  a.step_base_value = (long long)h->step;
  a.lr = h->cfg.lr;
  a.b1 = h->cfg.beta1;
  a.b2 = h->cfg.beta2;
  a.eps = h->cfg.eps;
  a.wd = h->cfg.weight_decay;
  a.grad_divisor = grad_divisor;
  launch_adamw(a, h->ctx.num_sms, s);
  MMN_CUDA_TRY(cudaGetLastError());
  if (!direct) MMN_CUDA_TRY(copy_out(param, p, numel, mem, s));
  if (mem == MMN_MEM_HOST) MMN_CUDA_TRY(cudaStreamSynchronize(s));
  return MMN_OK;
}

extern "C" int mmn_adamw_get_step(const mmn_adamw_t* h, uint64_t* step) {
  if (!h || !step) return fail(MMN_E_INVALID, "null argument");
  *step = h->step;
  return MMN_OK;
}

extern "C" int mmn_adamw_set_step(mmn_adamw_t* h, uint64_t step) {
  if (!h) return fail(MMN_E_INVALID, "null handle");
  h->step = step;
  return MMN_OK;
}

extern "C" int mmn_adamw_export_state(mmn_adamw_t* h, uint64_t id, int which, float* buf,
                                      int64_t numel, int mem) {
  if (!h || !buf || (which != 0 && which != 1)) return fail(MMN_E_INVALID, "bad argument");
  auto it = h->state.find(id);
  if (it == h->state.end()) return fail(MMN_E_STATE, "no state for this id");
  if (it->second.numel != numel) return fail(MMN_E_SHAPE, "numel differs from the state");
  DeviceGuard g(h->ctx.device);
  MMN_CUDA_TRY(copy_out(buf, which == 0 ? it->second.m : it->second.v, numel, mem, h->ctx.stream));
  MMN_CUDA_TRY(cudaStreamSynchronize(h->ctx.stream));
  return MMN_OK;
}

extern "C" int mmn_adamw_import_state(mmn_adamw_t* h, uint64_t id, int which, const float* buf,
                                      int64_t numel, int mem) {
  if (!h || !buf || (which != 0 && which != 1)) return fail(MMN_E_INVALID, "bad argument");
  DeviceGuard g(h->ctx.device);
  auto it = h->state.find(id);
  mmn_adamw::State* st = nullptr;
  if (it == h->state.end()) {
    const int64_t shape1[1] = {numel};
    int rc = adamw_state(h, id, shape1, 1, numel, &st);
    if (rc != MMN_OK) return rc;
  } else {
    st = &it->second;
    if (st->numel != numel) return fail(MMN_E_SHAPE, "numel differs from the state");
  }
  MMN_CUDA_TRY(copy_in(which == 0 ? st->m : st->v, buf, numel, mem, h->ctx.stream));
  MMN_CUDA_TRY(cudaStreamSynchronize(h->ctx.stream));
  return MMN_OK;
}

// ====================================================================== Muon
struct mmn_muon {
  Ctx ctx;
  mmn_muon_config cfg;
  int ns_mode = kNsReference;
  struct Vel {
    float* vel = nullptr;
    int rows = 0, cols = 0;
  };
  std::unordered_map<uint64_t, Vel> vel;
  std::map<std::pair<int, int>, NsClass> classes;
  Scratch sp, sg, spart, smeta, svel;
  bool gemm_ready = false;
};

static int muon_class(mmn_muon* h, int n, int m, NsClass** out) {
  if (!h->gemm_ready) {
    std::string e = ns_gemm_setup();
    if (!e.empty()) return fail(MMN_E_CUDA, e);
    h->gemm_ready = true;
  }
  auto key = std::make_pair(n, m);
  auto it = h->classes.find(key);
  if (it == h->classes.end()) {
    NsClass c;
    std::string e =
        ns_class_init(c, n, m, 1, nullptr, ns_elem_bytes(h->ns_mode), ns_planes(h->ns_mode));
    if (!e.empty()) {
      ns_class_free(c);  // (frees the buffers a failed init may already hold)
      return fail(MMN_E_CUDA, e);
    }
    it = h->classes.emplace(key, c).first;
  }
  *out = &it->second;
  return MMN_OK;
}

// Muon::step_matrix on device buffers: p (rows x cols) -= lr_scale * NS(u).
// vel may be fresh (read as zero). All work is enqueued on the handle's stream.
static int muon_run(mmn_muon* h, float* p, const float* g, float* vel, int rows, int cols,
                    float grad_divisor, float momentum, int nesterov, float lr_scale,
                    int fresh) {
  const int n = rows < cols ? rows : cols, m = rows < cols ? cols : rows;
  NsClass* c = nullptr;
  int rc = muon_class(h, n, m, &c);
  if (rc != MMN_OK) return rc;
  cudaStream_t s = h->ctx.stream;
  const int tiles = ((rows + 63) / 64) * ((cols + 63) / 64);
  if ((rc = h->spart.ensure((size_t)tiles * 4)) != MMN_OK) return rc;
  if ((rc = h->smeta.ensure(sizeof(MuonMat) + 2 * sizeof(MuonClassPtr) + 256)) != MMN_OK) return rc;
  const int steps = h->cfg.ns_steps;
  const int final_buf = steps % 2;
  struct {
    MuonMat mat;
    MuonClassPtr cls[2];
  } meta;
  memset(&meta, 0, sizeof(meta));
  meta.mat.off = 0;
  meta.mat.rows = rows;
  meta.mat.cols = cols;
  meta.mat.transposed = rows > cols;
  meta.mat.lr_scale = lr_scale;
  meta.mat.norm_idx = 0;
  meta.cls[0].x = c->x[0];
  meta.cls[0].bstride = (long long)c->n * c->ld_x;
  meta.cls[0].ld = c->ld_x;
  meta.cls[1] = meta.cls[0];
  meta.cls[1].x = c->x[final_buf];
  MMN_CUDA_TRY(cudaMemcpyAsync(h->smeta.ptr, &meta, sizeof(meta), cudaMemcpyHostToDevice, s));
  uint8_t* base = static_cast<uint8_t*>(h->smeta.ptr);
  MuonArgs a{};
  a.p = p;
  a.g = g;
  a.vel = vel;
  a.mats = reinterpret_cast<const MuonMat*>(base + offsetof(decltype(meta), mat));
  a.nmat = 1;
  a.total_tiles = tiles;
  a.cls = reinterpret_cast<const MuonClassPtr*>(base + offsetof(decltype(meta), cls));
  a.partials = static_cast<float*>(h->spart.ptr);
  a.norms = c->norms;
  a.momentum = momentum;
  a.nesterov = nesterov;
  a.grad_divisor = grad_divisor;
  a.fresh_state = fresh;
  a.apply_divides_norm = steps == 0;
  a.x_mode = h->ns_mode == kNsFp32 ? 2 : (h->ns_mode == kNsTf32 ? 1 : 0);
  a.norm_scalar_rows = (rows > cols ? rows : cols) % 8 != 0;
  launch_muon_momentum(a, h->ctx.num_sms, s);
  const long long numel = (long long)rows * cols;
  launch_muon_norms(a, s, ref_norm_cluster(numel, numel, 1, h->ctx.num_sms));
  MMN_CUDA_TRY(cudaGetLastError());
  std::string err;
  if (ns_class_run(*c, steps, h->ns_mode, h->ctx.status, h->ctx.num_sms, s, &err) < 0)
    return fail(MMN_E_CUDA, err);
  a.cls = reinterpret_cast<const MuonClassPtr*>(base + offsetof(decltype(meta), cls)) + 1;
  launch_muon_apply(a, h->ctx.num_sms, s);
  MMN_CUDA_TRY(cudaGetLastError());
  return MMN_OK;
}

extern "C" int mmn_muon_create(const mmn_muon_config* cfg, int ns_mode, int device, void* stream,
                               mmn_muon_t** out) {
  if (!out) return fail(MMN_E_INVALID, "out is null");
  *out = nullptr;
  if (ns_mode < MMN_NS_REFERENCE || ns_mode > MMN_NS_FP32)
    return fail(MMN_E_INVALID, "unknown ns_mode");
  mmn_muon_config c = cfg ? *cfg : mmn_muon_config_default();
  if (c.ns_steps < 0) return fail(MMN_E_INVALID, "ns_steps must be >= 0");
  auto* h = new mmn_muon();
  h->cfg = c;
  h->ns_mode = ns_mode;
  int rc = h->ctx.init(device, stream);
  if (rc != MMN_OK) {
    delete h;
    return rc;
  }
  *out = h;
  return MMN_OK;
}

extern "C" int mmn_muon_destroy(mmn_muon_t* h) {
  if (!h) return MMN_OK;
  DeviceGuard g(h->ctx.device);
  cudaStreamSynchronize(h->ctx.stream);
  for (auto& kv : h->vel) cudaFree(kv.second.vel);
  for (auto& kv : h->classes) ns_class_free(kv.second);
  h->sp.release();
  h->sg.release();
  h->spart.release();
  h->smeta.release();
  h->svel.release();
  h->ctx.release();
  delete h;
  return MMN_OK;
}

extern "C" int mmn_muon_step_matrix(mmn_muon_t* h, uint64_t id, float* param, const float* grad,
                                    const int64_t* shape, int ndim, float grad_divisor, int mem) {
  if (!h || !param || !grad) return fail(MMN_E_INVALID, "null handle, param or grad");
  if (mem != MMN_MEM_HOST && mem != MMN_MEM_DEVICE) return fail(MMN_E_INVALID, "bad mem kind");
  if (ndim != 2 || !shape)
    return fail(MMN_E_SHAPE, "Muon::step_matrix needs a 2-D param (the reference panics otherwise)");
  if (shape[0] < 1 || shape[1] < 1 || shape[0] > (1 << 30) || shape[1] > (1 << 30))
    return fail(MMN_E_SHAPE, "matrix dimensions out of range");
  if (!(grad_divisor > 0.0f)) return fail(MMN_E_INVALID, "grad_divisor must be > 0");
  const int rows = (int)shape[0], cols = (int)shape[1];
  const int64_t numel = (int64_t)rows * cols;
  DeviceGuard g(h->ctx.device);
  if (mem == MMN_MEM_DEVICE) {
    int rc0;
    if ((rc0 = check_device_ptr(param, h->ctx.device, "param")) != MMN_OK) return rc0;
    if ((rc0 = check_device_ptr(grad, h->ctx.device, "grad")) != MMN_OK) return rc0;
  }
  cudaStream_t s = h->ctx.stream;
  auto it = h->vel.find(id);
  if (it == h->vel.end()) {
    mmn_muon::Vel v;
    v.rows = rows;
    v.cols = cols;
    MMN_CUDA_TRY(cudaMalloc(&v.vel, (size_t)numel * 4));
    const cudaError_t e = cudaMemsetAsync(v.vel, 0, (size_t)numel * 4, s);
    if (e != cudaSuccess) {
      cudaFree(v.vel);
      return cuda_fail(e, "cudaMemsetAsync");
    }
    it = h->vel.emplace(id, v).first;
  } else if (it->second.rows != rows || it->second.cols != cols) {
    return fail(MMN_E_SHAPE, "grad shape differs from the velocity registered for this id");
  }
  float* p = param;
  const float* gp = grad;
  int rc;
  if (mem == MMN_MEM_HOST) {
    if ((rc = h->sp.ensure((size_t)numel * 4)) != MMN_OK) return rc;
    if ((rc = h->sg.ensure((size_t)numel * 4)) != MMN_OK) return rc;
    p = static_cast<float*>(h->sp.ptr);
    MMN_CUDA_TRY(copy_in(p, param, numel, mem, s));
    MMN_CUDA_TRY(copy_in(static_cast<float*>(h->sg.ptr), grad, numel, mem, s));
    gp = static_cast<const float*>(h->sg.ptr);
  }
  const float scale = sqrtf((float)rows / (float)cols);  // lib.rs:169-171
  const float lr_scale = h->cfg.lr * scale;               // lib.rs:173, (lr*scale)*u
  rc = muon_run(h, p, gp, it->second.vel, rows, cols, grad_divisor, h->cfg.momentum,
                h->cfg.nesterov, lr_scale, 0);
  if (rc != MMN_OK) return rc;
  if (mem == MMN_MEM_HOST) {
    MMN_CUDA_TRY(copy_out(param, p, numel, mem, s));
    return h->ctx.check_status();
  }
  return MMN_OK;
}

extern "C" int mmn_muon_export_velocity(mmn_muon_t* h, uint64_t id, float* buf, int64_t numel,
                                        int mem) {
  if (!h || !buf) return fail(MMN_E_INVALID, "null argument");
  auto it = h->vel.find(id);
  if (it == h->vel.end()) return fail(MMN_E_STATE, "no velocity for this id");
  if ((int64_t)it->second.rows * it->second.cols != numel) return fail(MMN_E_SHAPE, "numel differs");
  DeviceGuard g(h->ctx.device);
  MMN_CUDA_TRY(copy_out(buf, it->second.vel, numel, mem, h->ctx.stream));
  MMN_CUDA_TRY(cudaStreamSynchronize(h->ctx.stream));
  return MMN_OK;
}

extern "C" int mmn_muon_import_velocity(mmn_muon_t* h, uint64_t id, const float* buf,
                                        int64_t numel, int mem) {
  if (!h || !buf) return fail(MMN_E_INVALID, "null argument");
  auto it = h->vel.find(id);
  if (it == h->vel.end()) return fail(MMN_E_STATE, "step or register the id first");
  if ((int64_t)it->second.rows * it->second.cols != numel) return fail(MMN_E_SHAPE, "numel differs");
  DeviceGuard g(h->ctx.device);
  MMN_CUDA_TRY(copy_in(it->second.vel, buf, numel, mem, h->ctx.stream));
  MMN_CUDA_TRY(cudaStreamSynchronize(h->ctx.stream));
  return MMN_OK;
}

// Declares a velocity for an id without stepping (so it can be imported).
extern "C" int mmn_muon_register(mmn_muon_t* h, uint64_t id, const int64_t* shape, int ndim) {
  if (!h || ndim != 2 || !shape) return fail(MMN_E_INVALID, "2-D shape required");
  if (shape[0] < 1 || shape[1] < 1 || shape[0] > (1 << 30) || shape[1] > (1 << 30))
    return fail(MMN_E_SHAPE, "matrix dimensions out of range");
  auto it = h->vel.find(id);
  if (it != h->vel.end()) {
    if (it->second.rows != shape[0] || it->second.cols != shape[1])
      return fail(MMN_E_SHAPE, "shape differs from the velocity registered for this id");
    return MMN_OK;
  }
  DeviceGuard g(h->ctx.device);
  mmn_muon::Vel v;
  v.rows = (int)shape[0];
  v.cols = (int)shape[1];
  const size_t bytes = (size_t)v.rows * v.cols * 4;
  MMN_CUDA_TRY(cudaMalloc(&v.vel, bytes));
  const cudaError_t e = cudaMemset(v.vel, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(v.vel);
    return cuda_fail(e, "cudaMemset");
  }
  h->vel.emplace(id, v);
  return MMN_OK;
}

extern "C" int mmn_newton_schulz5(const float* g, const int64_t* shape, int ndim, int steps,
                                  int ns_mode, float* out, int device, void* stream, int mem) {
  if (!g || !out) return fail(MMN_E_INVALID, "null input or output");
  if (steps < 0) return fail(MMN_E_INVALID, "steps must be >= 0");
  int rc;
  const int64_t len = shape_numel(shape, ndim, &rc);
  if (rc != MMN_OK) return rc;
  int64_t rows, cols;
  if (ndim == 2) {
    rows = shape[0];
    cols = shape[1];
  } else {
    // lib.rs:93-99: side = ceil(sqrt(len as f32)); zero-padded row-major.
    const int64_t side = (int64_t)ceilf(sqrtf((float)len));
    rows = cols = side;
  }
  if (rows < 1 || cols < 1) return fail(MMN_E_SHAPE, "empty matrix");
  if (rows > (1 << 30) || cols > (1 << 30) || rows * cols < len)
    return fail(MMN_E_SHAPE, "matrix dimensions out of range");
  mmn_muon_config c = mmn_muon_config_default();
  c.ns_steps = steps;
  mmn_muon_t* h = nullptr;
  if ((rc = mmn_muon_create(&c, ns_mode, device, stream, &h)) != MMN_OK) return rc;
  DeviceGuard guard(device);
  cudaStream_t s = h->ctx.stream;
  const int64_t numel = rows * cols;
  auto run = [&]() -> int {
    int r;
    if ((r = h->sp.ensure((size_t)numel * 4)) != MMN_OK) return r;
    if ((r = h->sg.ensure((size_t)numel * 4)) != MMN_OK) return r;
    if ((r = h->svel.ensure((size_t)numel * 4)) != MMN_OK) return r;
    float* pd = static_cast<float*>(h->sp.ptr);
    float* gd = static_cast<float*>(h->sg.ptr);
    MMN_CUDA_TRY(cudaMemsetAsync(pd, 0, (size_t)numel * 4, s));
    MMN_CUDA_TRY(cudaMemsetAsync(gd, 0, (size_t)numel * 4, s));
    MMN_CUDA_TRY(copy_in(gd, g, len, mem, s));
    // momentum 0, no Nesterov: u = g exactly; p = 0 - (-1 * O) = O.
    r = muon_run(h, pd, gd, static_cast<float*>(h->svel.ptr), (int)rows, (int)cols, 1.0f, 0.0f,
                 0, -1.0f, 1);
    if (r != MMN_OK) return r;
    MMN_CUDA_TRY(copy_out(out, pd, numel, mem, s));
    return h->ctx.check_status();
  };
  rc = run();
  mmn_muon_destroy(h);
  return rc;
}

extern "C" int mmn_newton_schulz_iteration(const float* x, int64_t n, int64_t m, float x_norm,
                                           int ns_mode, float* a_out, float* a2_out,
                                           float* x_next, int device) {
  if (!x) return fail(MMN_E_INVALID, "null input");
  if (n < 1 || m < n || m > (1 << 30)) return fail(MMN_E_SHAPE, "need 1 <= n <= m");
  if (ns_mode < MMN_NS_REFERENCE || ns_mode > MMN_NS_FP32)
    return fail(MMN_E_INVALID, "unknown ns_mode");
  Ctx ctx;
  int rc = ctx.init(device, nullptr);
  if (rc != MMN_OK) return rc;
  DeviceGuard guard(device);
  std::string e = ns_gemm_setup();
  if (!e.empty()) {
    ctx.release();
    return fail(MMN_E_CUDA, e);
  }
  NsClass c;
  const bool f32 = ns_mode == MMN_NS_TF32 || ns_mode == MMN_NS_FP32;
  const bool split = ns_mode == MMN_NS_FP32;
  e = ns_class_init(c, (int)n, (int)m, 1, nullptr, ns_elem_bytes(ns_mode), ns_planes(ns_mode));
  if (!e.empty()) {
    ns_class_free(c);
    ctx.release();
    return fail(MMN_E_OOM, e);
  }
  auto run = [&]() -> int {
    if (split) {
      // fp32 mode: the hi and lo tf32 planes of x, one matrix item each
      const size_t plane = (size_t)n * c.ld_x;
      std::vector<float> hx(2 * plane, 0.0f);
      for (int64_t i = 0; i < n; ++i)
        for (int64_t j = 0; j < m; ++j) {
          const float v = x[i * m + j], hi = host_tf32_round(v);
          hx[(size_t)i * c.ld_x + j] = hi;
          hx[plane + (size_t)i * c.ld_x + j] = host_tf32_round(v - hi);
        }
      MMN_CUDA_TRY(cudaMemcpy(c.x[0], hx.data(), hx.size() * 4, cudaMemcpyHostToDevice));
    } else if (f32) {
      std::vector<float> hx((size_t)n * c.ld_x, 0.0f);
      for (int64_t i = 0; i < n; ++i)
        for (int64_t j = 0; j < m; ++j) hx[(size_t)i * c.ld_x + j] = host_tf32_round(x[i * m + j]);
      MMN_CUDA_TRY(cudaMemcpy(c.x[0], hx.data(), hx.size() * 4, cudaMemcpyHostToDevice));
    } else {
      std::vector<__nv_bfloat16> hx((size_t)n * c.ld_x, __float2bfloat16_rn(0.0f));
      for (int64_t i = 0; i < n; ++i)
        for (int64_t j = 0; j < m; ++j)
          hx[(size_t)i * c.ld_x + j] = __float2bfloat16_rn(x[i * m + j]);
      MMN_CUDA_TRY(cudaMemcpy(c.x[0], hx.data(), hx.size() * 2, cudaMemcpyHostToDevice));
    }
    MMN_CUDA_TRY(cudaMemcpy(c.norms, &x_norm, sizeof(float), cudaMemcpyHostToDevice));
    std::string err;
    if (ns_class_run(c, 1, ns_mode, ctx.status, ctx.num_sms, ctx.stream, &err) < 0)
      return fail(MMN_E_CUDA, err);
    int r = ctx.check_status();
    if (r != MMN_OK) return r;
    auto fetch = [&](const void* src, int64_t rows, int64_t cols, int ld, float* dst) -> int {
      if (!dst) return MMN_OK;
      if (f32) {
        // (fp32 mode: hi plane then lo plane; the value is their sum)
        const size_t plane = (size_t)rows * ld;
        std::vector<float> h(plane * (split ? 2 : 1));
        MMN_CUDA_TRY(cudaMemcpy(h.data(), src, h.size() * 4, cudaMemcpyDeviceToHost));
        for (int64_t i = 0; i < rows; ++i)
          for (int64_t j = 0; j < cols; ++j) {
            const size_t k = (size_t)i * ld + j;
            dst[i * cols + j] = split ? h[k] + h[plane + k] : h[k];
          }
        return MMN_OK;
      }
      std::vector<__nv_bfloat16> h((size_t)rows * ld);
      MMN_CUDA_TRY(cudaMemcpy(h.data(), src, h.size() * 2, cudaMemcpyDeviceToHost));
      for (int64_t i = 0; i < rows; ++i)
        for (int64_t j = 0; j < cols; ++j) dst[i * cols + j] = __bfloat162float(h[(size_t)i * ld + j]);
      return MMN_OK;
    };
    if ((r = fetch(c.a, n, n, c.ld_a, a_out)) != MMN_OK) return r;
    if ((r = fetch(c.a2, n, n, c.ld_a, a2_out)) != MMN_OK) return r;
    return fetch(c.x[1], n, m, c.ld_x, x_next);
  };
  rc = run();
  ns_class_free(c);
  ctx.release();
  return rc;
}

// ==================================================================== Hybrid
struct mmn_hybrid {
  mmn_adamw_t* adamw = nullptr;
  mmn_muon_t* muon = nullptr;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  int device = 0;
};

extern "C" int mmn_hybrid_create(const mmn_muon_config* muon, const mmn_adamw_config* adamw,
                                 int ns_mode, int device, void* stream, mmn_hybrid_t** out) {
  if (!out) return fail(MMN_E_INVALID, "out is null");
  *out = nullptr;
  auto* h = new mmn_hybrid();
  h->device = device;
  int rc = MMN_OK;
  if (!stream) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
      cudaGetLastError();
      delete h;
      return fail(MMN_E_NO_DEVICE, "GPU missing, but CUDA was requested.");
    }
    DeviceGuard g(device);
    if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess) {
      delete h;
      return fail(MMN_E_CUDA, "cudaStreamCreate failed");
    }
    h->own_stream = true;
    stream = h->stream;
  }
  rc = mmn_adamw_create(adamw, device, stream, &h->adamw);
  if (rc == MMN_OK) rc = mmn_muon_create(muon, ns_mode, device, stream, &h->muon);
  if (rc != MMN_OK) {
    mmn_adamw_destroy(h->adamw);
    if (h->own_stream) cudaStreamDestroy(h->stream);
    delete h;
    return rc;
  }
  *out = h;
  return MMN_OK;
}

extern "C" int mmn_hybrid_destroy(mmn_hybrid_t* h) {
  if (!h) return MMN_OK;
  mmn_adamw_destroy(h->adamw);
  mmn_muon_destroy(h->muon);
  if (h->own_stream) {
    DeviceGuard g(h->device);
    cudaStreamDestroy(h->stream);
  }
  delete h;
  return MMN_OK;
}

extern "C" int mmn_hybrid_step(mmn_hybrid_t* h, uint64_t id, float* param, const float* grad,
                               const int64_t* shape, int ndim, int route, float grad_divisor,
                               int mem) {
  if (!h) return fail(MMN_E_INVALID, "null handle");
  if (route == MMN_ROUTE_AUTO) route = mmn_hybrid_classify_param(shape, ndim);
  if (route == MMN_ROUTE_MUON)
    return mmn_muon_step_matrix(h->muon, id, param, grad, shape, ndim, grad_divisor, mem);
  if (route == MMN_ROUTE_ADAMW)
    return mmn_adamw_step_param(h->adamw, id, param, grad, shape, ndim, grad_divisor, mem);
  return fail(MMN_E_INVALID, "unknown route");
}

extern "C" mmn_adamw_t* mmn_hybrid_adamw(mmn_hybrid_t* h) { return h ? h->adamw : nullptr; }
extern "C" mmn_muon_t* mmn_hybrid_muon(mmn_hybrid_t* h) { return h ? h->muon : nullptr; }

// ============================================== grad reduction, caller's buffers
namespace {

// Device (or managed) memory of `device`, or of a peer GPU that `device` can
// reach, with peer access enabled here: a source of mmn_grad_reduce or a flag
// of mmn_grad_nonfinite_scan.
int check_reachable(const void* p, int device, const std::string& what) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return fail(MMN_E_INVALID, what + ": not a CUDA pointer");
  }
  if (at.type == cudaMemoryTypeManaged) return MMN_OK;
  if (at.type != cudaMemoryTypeDevice)
    return fail(MMN_E_INVALID, what + ": host memory where device memory is needed");
  if (at.device == device) return MMN_OK;
  int can = 0;
  if (cudaDeviceCanAccessPeer(&can, device, at.device) != cudaSuccess || !can) {
    cudaGetLastError();
    return fail(MMN_E_INVALID, what + ": memory of device " + std::to_string(at.device) +
                                   ", which device " + std::to_string(device) + " cannot reach");
  }
  const cudaError_t e = cudaDeviceEnablePeerAccess(at.device, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
  } else if (e != cudaSuccess) {
    return cuda_fail(e, "cudaDeviceEnablePeerAccess");
  }
  return MMN_OK;
}

// The device checks of the caller-buffer entry points: a usable sm_100 GPU.
int percall_device(int device, int* sms) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    return fail(MMN_E_NO_DEVICE, "GPU missing, but CUDA was requested.");
  }
  if (device < 0 || device >= count) return fail(MMN_E_INVALID, "device ordinal out of range");
  int major = 0, minor = 0;
  MMN_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
  MMN_CUDA_TRY(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
  MMN_CUDA_TRY(cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, device));
  if (major != 10 || minor != 0)
    return fail(MMN_E_NO_DEVICE, "this library is built for sm_100a (B200) devices only");
  return MMN_OK;
}

}  // namespace

extern "C" int mmn_grad_reduce(const void* const* src, int nsrc, void* dst, int64_t numel,
                               int dtype, int* nonfinite_flag, int device, void* stream) {
  if (!src || !dst) return fail(MMN_E_INVALID, "null source list or destination");
  if (nsrc < 2 || nsrc > kMaxRanks) return fail(MMN_E_INVALID, "nsrc must lie in [2, 8]");
  if (dtype != MMN_DTYPE_F32 && dtype != MMN_DTYPE_BF16)
    return fail(MMN_E_INVALID, "unknown dtype");
  if (numel < 0 || numel > (int64_t(1) << 60)) return fail(MMN_E_INVALID, "numel out of range");
  for (int k = 0; k < nsrc; ++k)
    if (!src[k]) return fail(MMN_E_INVALID, "null source pointer");
  const uintptr_t d0 = reinterpret_cast<uintptr_t>(dst);
  if (d0 % 16) return fail(MMN_E_INVALID, "dst is not 16-byte aligned");
  const uintptr_t bytes = (uintptr_t)numel * (dtype == MMN_DTYPE_BF16 ? 2u : 4u);
  for (int k = 0; k < nsrc; ++k) {
    const uintptr_t s0 = reinterpret_cast<uintptr_t>(src[k]);
    if (s0 % 16) return fail(MMN_E_INVALID, "a source is not 16-byte aligned");
    if (s0 != d0 && s0 < d0 + bytes && d0 < s0 + bytes)
      return fail(MMN_E_INVALID, "dst overlaps a source it does not equal");
  }
  if (nonfinite_flag && reinterpret_cast<uintptr_t>(nonfinite_flag) % 4)
    return fail(MMN_E_INVALID, "nonfinite_flag is not 4-byte aligned");
  int sms = 0, rc;
  if ((rc = percall_device(device, &sms)) != MMN_OK) return rc;
  DeviceGuard guard(device);
  if ((rc = check_device_ptr(dst, device, "dst")) != MMN_OK) return rc;
  if (nonfinite_flag && (rc = check_device_ptr(nonfinite_flag, device, "nonfinite_flag")) != MMN_OK)
    return rc;
  for (int k = 0; k < nsrc; ++k)
    if ((rc = check_reachable(src[k], device, "src[" + std::to_string(k) + "]")) != MMN_OK)
      return rc;
  if (numel == 0) return MMN_OK;
  GradReduceArgs a{};
  a.world = nsrc;
  a.bf16 = dtype == MMN_DTYPE_BF16;
  a.scan = nonfinite_flag != nullptr;
  for (int k = 0; k < nsrc; ++k) {
    a.src[k] = src[k];
    a.skip_flags[k] = nonfinite_flag;  // one flag: every "rank" slot points at it
  }
  a.dst = dst;
  a.begin = 0;
  a.end = numel;
  launch_grad_reduce(a, sms, static_cast<cudaStream_t>(stream));
  MMN_CUDA_TRY(cudaGetLastError());
  return MMN_OK;
}

extern "C" int mmn_grad_nonfinite_scan(const void* grads, int64_t numel, int dtype,
                                       int* const* flags, int nflags, int device, void* stream) {
  if (!grads || !flags) return fail(MMN_E_INVALID, "null grads or flag list");
  if (nflags < 1 || nflags > kMaxRanks) return fail(MMN_E_INVALID, "nflags must lie in [1, 8]");
  if (dtype != MMN_DTYPE_F32 && dtype != MMN_DTYPE_BF16)
    return fail(MMN_E_INVALID, "unknown dtype");
  if (numel < 0 || numel > (int64_t(1) << 60)) return fail(MMN_E_INVALID, "numel out of range");
  if (reinterpret_cast<uintptr_t>(grads) % 16) return fail(MMN_E_INVALID, "grads is not 16-byte aligned");
  for (int k = 0; k < nflags; ++k) {
    if (!flags[k]) return fail(MMN_E_INVALID, "null flag pointer");
    if (reinterpret_cast<uintptr_t>(flags[k]) % 4)
      return fail(MMN_E_INVALID, "a flag is not 4-byte aligned");
  }
  int sms = 0, rc;
  if ((rc = percall_device(device, &sms)) != MMN_OK) return rc;
  DeviceGuard guard(device);
  if ((rc = check_device_ptr(grads, device, "grads")) != MMN_OK) return rc;
  for (int k = 0; k < nflags; ++k)
    if ((rc = check_reachable(flags[k], device, "flags[" + std::to_string(k) + "]")) != MMN_OK)
      return rc;
  if (numel == 0) return MMN_OK;
  RankFlags f{};
  f.n = nflags;
  for (int k = 0; k < nflags; ++k) f.flag[k] = flags[k];
  const bool bf = dtype == MMN_DTYPE_BF16;
  launch_nonfinite_scan_ranks(bf ? nullptr : static_cast<const float*>(grads), bf ? 0 : numel,
                              bf ? static_cast<const __nv_bfloat16*>(grads) : nullptr,
                              bf ? numel : 0, f, sms, static_cast<cudaStream_t>(stream));
  MMN_CUDA_TRY(cudaGetLastError());
  return MMN_OK;
}
