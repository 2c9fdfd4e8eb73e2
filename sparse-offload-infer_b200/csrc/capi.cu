// C ABI entry points (include/soinfer_b200.h): argument validation with the
// reference binding's preconditions (csrc/bindings.cpp:176-559), then the
// sm_100a launchers.  Nothing here aborts; failures return a status and set
// the thread's last-error message.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/soinfer_b200.h"
#include "capi_util.h"
#include "kernels.h"

namespace soinfer {

namespace {
thread_local std::string g_last_error;
}

int set_error(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int cuda_result(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return SOINFER_OK;
  (void)cudaGetLastError();  // clear a non-sticky launch error
  return set_error(SOINFER_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

const char* last_error() { return g_last_error.c_str(); }

}  // namespace soinfer

using namespace soinfer;

#define REQUIRE(cond, ...)                                               \
  do {                                                                   \
    if (!(cond)) return set_error(SOINFER_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
  } while (0)

namespace {

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
inline const half* as_half(const soinfer_half* p) { return reinterpret_cast<const half*>(p); }
inline half* as_half(soinfer_half* p) { return reinterpret_cast<half*>(p); }
inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }
inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t int4_row_bytes(int64_t K) { return cdiv(K, 8) * 4; }

int check_int4_layout(const char* name, int64_t K, int64_t group_size, int64_t num_groups) {
  REQUIRE(K >= 1, "%s: K must be >= 1", name);
  REQUIRE(group_size >= 1 && group_size % 8 == 0, "%s: group_size must be a positive multiple of 8", name);
  REQUIRE(num_groups == cdiv(K, group_size),
          "%s: scale's num_groups must be ceil(K/group_size) for the given K and group_size, got %lld but expected %lld",
          name, (long long)num_groups, (long long)cdiv(K, group_size));
  return SOINFER_OK;
}

}  // namespace

extern "C" {

int soinfer_abi_version(void) { return 1; }

const char* soinfer_last_error(void) { return soinfer::last_error(); }

const char* soinfer_status_string(int status) {
  switch (status) {
    case SOINFER_OK: return "SOINFER_OK";
    case SOINFER_ERR_INVALID_ARGUMENT: return "SOINFER_ERR_INVALID_ARGUMENT";
    case SOINFER_ERR_CUDA: return "SOINFER_ERR_CUDA";
    case SOINFER_ERR_UNSUPPORTED: return "SOINFER_ERR_UNSUPPORTED";
    case SOINFER_ERR_HOST: return "SOINFER_ERR_HOST";
  }
  return "SOINFER_ERR_UNKNOWN";
}

int soinfer_device_errors(int* flags) {
  REQUIRE(flags, "device_errors: null flags");
  *flags = 0;
  int f = 0;
  if (int st = cuda_result(read_and_clear_gemv_w4_error(&f), "device_errors")) return st;
  *flags |= f;
  if (int st = cuda_result(read_and_clear_gemv_batch_error(&f), "device_errors")) return st;
  *flags |= f;
  if (int st = cuda_result(read_and_clear_tp_error(&f), "device_errors")) return st;
  *flags |= f;
  if (int st = cuda_result(read_and_clear_gemm_w4_error(&f), "device_errors")) return st;
  *flags |= f;
  if (int st = cuda_result(read_and_clear_gemv_stream_error(&f), "device_errors")) return st;
  *flags |= f;
  if (int st = cuda_result(read_and_clear_decode_fused_error(&f), "device_errors")) return st;
  *flags |= f;
  return SOINFER_OK;
}

int64_t soinfer_gemv_batch_workspace_bytes(int64_t num_tasks) {
  if (num_tasks < 0 || num_tasks > kMaxBatchTasks) return 0;
  return gemv_batch_workspace_bytes(num_tasks);
}

// True if task a waits, directly or through a chain of deps, for task b.
static bool waits_for(const soinfer_gemv_task* tasks, int64_t a, int64_t b) {
  for (int64_t d = tasks[a].dep; d >= 0; d = tasks[d].dep)
    if (d == b) return true;
  return false;
}

// The streaming kernel serves a batch of plain GEMVs (no epilogue or
// prologue; a task may wait for an earlier one) that is large enough to give
// every warp of the GPU at least two units.  A task's x may overlap another
// task's y, and two tasks' y may overlap, only when one of the two waits for
// the other (read after write, write after read, write after write).
static bool stream_eligible(const soinfer_gemv_task* tasks, int64_t n, int sms) {
  int64_t units = 0;
  for (int64_t i = 0; i < n; ++i) {
    const soinfer_gemv_task& t = tasks[i];
    if (t.residual || t.glu_gate || t.norm_weight || !t.y || !aligned(t.x, 8)) return false;
    units += cdiv(t.N, 16 * kStreamTiles);
  }
  if (units < 2LL * sms * kStreamWarps) return false;
  for (int64_t i = 0; i < n; ++i) {
    const uintptr_t ylo = reinterpret_cast<uintptr_t>(tasks[i].y), yhi = ylo + 2 * tasks[i].N;
    for (int64_t j = 0; j < n; ++j) {
      const uintptr_t xlo = reinterpret_cast<uintptr_t>(tasks[j].x), xhi = xlo + 2 * tasks[j].K;
      if (xlo < yhi && ylo < xhi && !(j != i && (waits_for(tasks, j, i) || waits_for(tasks, i, j)))) return false;
      if (j != i) {
        const uintptr_t zlo = reinterpret_cast<uintptr_t>(tasks[j].y), zhi = zlo + 2 * tasks[j].N;
        // two tasks writing the same rows: only when one waits for the other
        if (zlo < yhi && ylo < zhi && !(waits_for(tasks, j, i) || waits_for(tasks, i, j))) return false;
      }
    }
  }
  return true;
}

static int gemv_batch_common(const char* name, const PeerSet* peers, const soinfer_gemv_task* tasks,
                             int64_t num_tasks, void* workspace, int64_t workspace_bytes, void* stream) {
  REQUIRE(num_tasks >= 0 && num_tasks <= kMaxBatchTasks, "%s: num_tasks must be in [0, %d]", name, kMaxBatchTasks);
  if (num_tasks == 0) return SOINFER_OK;
  REQUIRE(tasks, "%s: null task list", name);
  bool fast = true;
  int npeer = 0, nnorm = 0;
  for (int64_t i = 0; i < num_tasks; ++i) {
    const soinfer_gemv_task& t = tasks[i];
    char tn[64];
    snprintf(tn, sizeof(tn), "%s[task %lld]", name, (long long)i);
    if (int st = check_int4_layout(tn, t.K, t.group_size, t.num_groups)) return st;
    REQUIRE(t.N >= 1, "%s: N must be >= 1", tn);
    REQUIRE(t.Wq && t.scale && t.x && (t.y || peers), "%s: null pointer", tn);
    REQUIRE(t.dep >= -1 && t.dep < i, "%s: dep must be -1 or an earlier task index", tn);
    if (!t.y) {  // the row-parallel task whose rows go to the peers' inboxes
      ++npeer;
      REQUIRE(npeer == 1, "%s: at most one task per batch may send its rows to the peers (y == NULL)", tn);
      REQUIRE(t.N * 2 <= peers->slot_bytes, "%s: N rows exceed the exchange slot", tn);
      REQUIRE(!t.glu_gate && !t.residual, "%s: a peer task takes no epilogue (the exchange adds the residual)", tn);
      REQUIRE(t.K % 128 == 0 && t.group_size % 128 == 0 && aligned(t.Wq, 16) && aligned(t.x, 16) &&
                  aligned(t.scale, 4),
              "%s: a peer task needs K and group_size multiples of 128 and 16-byte aligned rows / x", tn);
    }
    REQUIRE(!t.norm_out || (t.norm_weight && aligned(t.norm_out, 16)), "%s: norm_out needs norm_weight and 16-byte "
            "alignment", tn);
    if (t.norm_weight) {
      REQUIRE(t.K % 128 == 0 && t.group_size % 128 == 0 && aligned(t.norm_weight, 16) && t.norm_eps >= 0.f,
              "%s: a norm prologue needs K and group_size multiples of 128, a 16-byte aligned weight and eps >= 0",
              tn);
      ++nnorm;
    }
    for (int64_t j = 0; j < i; ++j) {  // an epilogue input made in this batch must share the row split
      if (tasks[j].y && (tasks[j].y == t.glu_gate || tasks[j].y == t.residual))
        REQUIRE(tasks[j].N == t.N, "%s: glu_gate / residual is task %lld's y but N differs", tn, (long long)j);
    }
    fast = fast && t.K % 128 == 0 && t.group_size % 128 == 0 && aligned(t.Wq, 16) && aligned(t.scale, 4) &&
           (t.num_groups % 4 != 0 || aligned(t.scale, 16)) && aligned(t.x, 16) && t.N < (1 << 30) &&
           t.K < (1 << 30);
  }
  cudaStream_t st = as_stream(stream);
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (fast && !peers && stream_eligible(tasks, num_tasks, sms)) {
    // a large list of independent GEMVs: the streaming kernel (gemv_stream.cu)
    static GemvStreamParams S;
    static std::mutex smu;
    std::lock_guard<std::mutex> lk(smu);
    S.num = (int)num_tasks;
    S.m = 1;
    for (int64_t i = 0; i < num_tasks; ++i) {
      const soinfer_gemv_task& t = tasks[i];
      S.tasks[i] = GemvStreamTask{t.Wq, t.scale, as_half(t.x), as_half(t.y), (int)t.N, (int)t.K,
                                  (int)t.num_groups, (int)(t.group_size / 128), (int)t.K, (int)t.N, (int)t.dep,
                                  0, 0, 0};
    }
    if (plan_gemv_stream(S, sms)) {
      const int64_t need = gemv_stream_workspace_bytes(num_tasks);
      REQUIRE(workspace && workspace_bytes >= need && aligned(workspace, 4),
              "%s: workspace too small (need %lld zeroed bytes)", name, (long long)need);
      return cuda_result(launch_gemv_stream(S, reinterpret_cast<int*>(workspace), st), name);
    }
  }
  if (fast) {
    static GemvBatchParams B;  // large: not on the stack
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    B.num = (int)num_tasks;
    if (peers) {
      B.peers = *peers;
    } else {
      B.peers = PeerSet{};
      B.peers.world = 0;
    }
    for (int64_t i = 0; i < num_tasks; ++i) {
      const soinfer_gemv_task& t = tasks[i];
      GemvBatchTask& d = B.tasks[i];
      d.W = t.Wq;
      d.S = t.scale;
      d.x = as_half(t.x);
      d.y = as_half(t.y);
      d.N = (int)t.N;
      d.K = (int)t.K;
      d.G = (int)t.num_groups;
      d.cpg = (int)(t.group_size / 128);
      d.dep = (int)t.dep;
      d.resid = as_half(t.residual);
      d.glu = as_half(t.glu_gate);
      d.peer = t.y ? 0 : 1;
      d.norm_w = as_half(t.norm_weight);
      d.eps = t.norm_eps;
      d.norm_out = as_half(t.norm_out);
    }
    if (plan_gemv_batch(B, sms)) {
      REQUIRE(workspace && workspace_bytes >= gemv_batch_workspace_bytes(num_tasks) && aligned(workspace, 4),
              "%s: workspace too small (need %lld zeroed bytes)", name, (long long)gemv_batch_workspace_bytes(num_tasks));
      return cuda_result(launch_gemv_batch(B, reinterpret_cast<int*>(workspace), st), name);
    }
  }
  // fallback: ordered single-GEMV launches (stream order satisfies every dep)
  REQUIRE(nnorm == 0, "%s: a norm prologue needs the persistent path (K, group size multiples of 128; rows per "
                      "CTA <= 128)", name);
  for (int64_t i = 0; i < num_tasks; ++i) {
    const soinfer_gemv_task& t = tasks[i];
    RowSource src;
    src.W = t.Wq;
    src.S = t.scale;
    src.rows1 = t.N;
    src.row_bytes = int4_row_bytes(t.K);
    src.num_groups = t.num_groups;
    if (!t.y) {
      const cudaError_t e = launch_gemv_w4_peer(src, as_half(t.x), t.N, t.K, t.group_size, *peers, st);
      if (e == cudaErrorNotSupported)
        return set_error(SOINFER_ERR_UNSUPPORTED, "%s: peer task shape outside the bulk GEMV path", name);
      if (int rc = cuda_result(e, name)) return rc;
      continue;
    }
    if (int rc = cuda_result(launch_gemv_w4(RowMode::kPlain, src, as_half(t.x), as_half(t.y), t.N, t.K, t.group_size, st),
                             name))
      return rc;
    if (t.glu_gate)
      if (int rc = cuda_result(launch_swiglu(as_half(t.glu_gate), as_half(t.y), nullptr, as_half(t.y), t.N, st), name))
        return rc;
    if (t.residual)
      if (int rc = cuda_result(launch_add_half(as_half(t.residual), as_half(t.y), as_half(t.y), t.N, st), name))
        return rc;
  }
  return SOINFER_OK;
}

int64_t soinfer_gemm_batch_workspace_bytes(void) { return gemv_stream_workspace_bytes(0); }

int soinfer_gemm_w4a16_batch(const soinfer_gemm_task* tasks, int64_t num_tasks, int64_t M, void* workspace,
                             int64_t workspace_bytes, void* stream) {
  const char* name = "gemm_w4a16_batch";
  REQUIRE(num_tasks >= 0 && num_tasks <= kMaxBatchTasks, "%s: num_tasks must be in [0, %d]", name, kMaxBatchTasks);
  REQUIRE(M >= 1 && M <= 8, "%s: M must be in [1, 8]", name);
  if (num_tasks == 0) return SOINFER_OK;
  REQUIRE(tasks, "%s: null task list", name);
  static GemvStreamParams S;
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  S.num = (int)num_tasks;
  S.m = (int)M;
  for (int64_t i = 0; i < num_tasks; ++i) {
    const soinfer_gemm_task& t = tasks[i];
    char tn[64];
    snprintf(tn, sizeof(tn), "%s[task %lld]", name, (long long)i);
    if (int st = check_int4_layout(tn, t.K, t.group_size, t.num_groups)) return st;
    REQUIRE(t.N >= 1 && t.N < (1 << 30) && t.K < (1 << 30), "%s: N must be in [1, 2^30)", tn);
    REQUIRE(t.Wq && t.scale && t.X && t.Y, "%s: null pointer", tn);
    REQUIRE(t.ldx >= t.K && t.ldy >= t.N && t.ldx < (1 << 30) && t.ldy < (1 << 30), "%s: ldx >= K, ldy >= N", tn);
    if (!(t.K % 128 == 0 && t.group_size % 128 == 0 && aligned(t.Wq, 16) && aligned(t.X, 16) && t.ldx % 8 == 0 &&
          aligned(t.scale, 4) && aligned(t.Y, 2)))
      return set_error(SOINFER_ERR_UNSUPPORTED, "%s: needs K and group_size multiples of 128, 16-byte aligned "
                       "Wq and X rows, 4-byte aligned scales", tn);
    S.tasks[i] = GemvStreamTask{t.Wq, t.scale, as_half(t.X), as_half(t.Y), (int)t.N, (int)t.K, (int)t.num_groups,
                                (int)(t.group_size / 128), (int)t.ldx, (int)t.ldy, -1, 0, 0, 0};
  }
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  REQUIRE(plan_gemv_stream(S, sms), "%s: batch too large", name);
  REQUIRE(workspace && workspace_bytes >= gemv_stream_workspace_bytes(0) && aligned(workspace, 4),
          "%s: workspace too small (need %lld zeroed bytes)", name, (long long)gemv_stream_workspace_bytes(0));
  return cuda_result(launch_gemv_stream(S, reinterpret_cast<int*>(workspace), as_stream(stream)), name);
}

int64_t soinfer_decode_fused_workspace_bytes(int64_t hidden, int64_t intermediate, int64_t num_heads,
                                             int64_t num_kv_heads, int64_t head_dim) {
  if (hidden < 1 || intermediate < 1 || num_heads < 1 || num_kv_heads < 1 || head_dim < 1) return 0;
  return decode_fused_workspace_bytes(hidden, intermediate, num_heads, num_kv_heads, head_dim);
}

int soinfer_decode_layers_fused(const soinfer_fused_layer* layers, int64_t num_layers, int64_t hidden,
                                int64_t intermediate, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                                int64_t group_size, int64_t max_seq, float eps, const float* cos_table,
                                const float* sin_table, const int32_t* pos_dev, soinfer_half* x, void* workspace,
                                int64_t workspace_bytes, void* stream) {
  const char* name = "decode_layers_fused";
  REQUIRE(layers && x && pos_dev && cos_table && sin_table && workspace, "%s: null pointer", name);
  REQUIRE(num_layers >= 1 && hidden >= 1 && intermediate >= 1 && num_heads >= 1 && num_kv_heads >= 1 &&
              max_seq >= 1 && max_seq < (1 << 30),
          "%s: sizes must be positive", name);
  if (num_layers > kFusedMaxLayers || head_dim != 128 || group_size != 128 || num_heads % num_kv_heads != 0 ||
      hidden % 128 != 0 || intermediate % 128 != 0 || hidden > (1 << 20) || intermediate > (1 << 20) ||
      num_heads > 1024)
    return set_error(SOINFER_ERR_UNSUPPORTED, "%s: needs head_dim 128, group size 128, hidden / intermediate "
                     "multiples of 128, num_heads a multiple of num_kv_heads, <= %d layers", name, kFusedMaxLayers);
  REQUIRE(aligned(x, 16) && aligned(workspace, 256), "%s: x 16-byte and workspace 256-byte aligned", name);
  static FusedDecodeParams P;  // ~10 KB: not on the stack
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  P.layers = (int)num_layers;
  P.H = (int)hidden;
  P.I = (int)intermediate;
  P.NQ = (int)num_heads;
  P.NKV = (int)num_kv_heads;
  P.HD = (int)head_dim;
  P.max_seq = max_seq;
  P.eps = eps;
  P.cos_t = cos_table;
  P.sin_t = sin_table;
  P.pos = pos_dev;
  P.x = as_half(x);
  for (int64_t i = 0; i < num_layers; ++i) {
    const soinfer_fused_layer& l = layers[i];
    FusedLayer& d = P.layer[i];
    for (int m = 0; m < 7; ++m) {
      REQUIRE(l.Wq[m] && l.scale[m], "%s[layer %lld]: null weight", name, (long long)i);
      if (!aligned(l.Wq[m], 16) || !aligned(l.scale[m], 16))
        return set_error(SOINFER_ERR_UNSUPPORTED, "%s[layer %lld]: weight rows and scales must be 16-byte aligned",
                         name, (long long)i);
      d.w[m] = l.Wq[m];
      d.s[m] = l.scale[m];
    }
    REQUIRE(l.input_norm && l.post_norm && l.q_norm && l.k_norm && l.k_cache && l.v_cache,
            "%s[layer %lld]: null norm weight or cache", name, (long long)i);
    REQUIRE(aligned(l.input_norm, 16) && aligned(l.post_norm, 16) && aligned(l.k_cache, 16) && aligned(l.v_cache, 16),
            "%s[layer %lld]: norm weights and caches must be 16-byte aligned", name, (long long)i);
    d.in_norm = as_half(l.input_norm);
    d.post_norm = as_half(l.post_norm);
    d.q_norm = as_half(l.q_norm);
    d.k_norm = as_half(l.k_norm);
    d.kc = as_half(l.k_cache);
    d.vc = as_half(l.v_cache);
  }
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t need = decode_fused_workspace_bytes(hidden, intermediate, num_heads, num_kv_heads, head_dim);
  REQUIRE(workspace_bytes >= need, "%s: workspace too small (need %lld bytes)", name, (long long)need);
  if (!plan_decode_fused(P, workspace, workspace_bytes, sms))
    return set_error(SOINFER_ERR_UNSUPPORTED, "%s: shape not served by the fused step (num_heads / num_kv_heads "
                     "in {1, 2, 4}, at most %d tiles per SM per phase, shared memory)", name, 16);
  return cuda_result(launch_decode_fused(P, sms, as_stream(stream)), name);
}

int soinfer_gemv_w4a16_batch(const soinfer_gemv_task* tasks, int64_t num_tasks, void* workspace,
                             int64_t workspace_bytes, void* stream) {
  return gemv_batch_common("gemv_w4a16_batch", nullptr, tasks, num_tasks, workspace, workspace_bytes, stream);
}

static int gemv_w4_plain(const char* name, const uint8_t* Wq, const float* scale, const soinfer_half* x,
                         soinfer_half* y, int64_t N, int64_t K, int64_t group_size, int64_t num_groups, void* stream,
                         uint32_t flags = 0) {
  if (int st = check_int4_layout(name, K, group_size, num_groups)) return st;
  REQUIRE(N >= 0, "%s: N must be >= 0", name);
  if (N == 0) return SOINFER_OK;
  REQUIRE(Wq && scale && x && y, "%s: null pointer", name);
  REQUIRE(aligned(Wq, 4) && aligned(x, 2) && aligned(y, 2) && aligned(scale, 4), "%s: misaligned pointer", name);
  RowSource src;
  src.W = Wq;
  src.S = scale;
  src.rows1 = N;
  src.row_bytes = int4_row_bytes(K);
  src.num_groups = num_groups;
  LaunchOpts opts;
  opts.pdl = (flags & SOINFER_FLAG_PDL) != 0;
  return cuda_result(
      launch_gemv_w4(RowMode::kPlain, src, as_half(x), as_half(y), N, K, group_size, as_stream(stream), opts), name);
}

int soinfer_gemv_w4a16_group_ex(const uint8_t* Wq, const float* scale, const soinfer_half* x, soinfer_half* y,
                                int64_t N, int64_t K, int64_t group_size, int64_t num_groups, uint32_t flags,
                                void* stream) {
  REQUIRE((flags & ~SOINFER_FLAG_PDL) == 0, "gemv_w4a16_group_ex: unknown flags 0x%x", flags);
  return gemv_w4_plain("gemv_w4a16_group_ex", Wq, scale, x, y, N, K, group_size, num_groups, stream, flags);
}

int soinfer_gemv_w4a16_group(const uint8_t* Wq, const float* scale, const soinfer_half* x, soinfer_half* y, int64_t N,
                             int64_t K, int64_t group_size, int64_t num_groups, void* stream) {
  return gemv_w4_plain("gemv_w4a16_group", Wq, scale, x, y, N, K, group_size, num_groups, stream);
}

int soinfer_gemv_w4a16_group_lop3(const uint8_t* Wq, const float* scale, const soinfer_half* x, soinfer_half* y,
                                  int64_t N, int64_t K, int64_t group_size, int64_t num_groups, void* stream) {
  return gemv_w4_plain("gemv_w4a16_group_lop3", Wq, scale, x, y, N, K, group_size, num_groups, stream);
}

int soinfer_gemv_w4a16_rows(const uint8_t* Wq, const float* scale, int64_t N, const int32_t* rows, int64_t num_sel,
                            const soinfer_half* x, soinfer_half* y, int64_t K, int64_t group_size, int64_t num_groups,
                            const soinfer_half* glu_gate, void* stream) {
  const char* name = "gemv_w4a16_rows";
  if (int st = check_int4_layout(name, K, group_size, num_groups)) return st;
  REQUIRE(num_sel >= 0 && N >= 0, "%s: sizes must be >= 0", name);
  if (num_sel == 0) return SOINFER_OK;
  REQUIRE(N >= 1, "%s: cannot select rows of an empty matrix", name);
  REQUIRE(Wq && scale && rows && x && y, "%s: null pointer", name);
  REQUIRE(aligned(Wq, 4) && aligned(rows, 4) && aligned(scale, 4), "%s: misaligned pointer", name);
  RowSource src;
  src.W = Wq;
  src.S = scale;
  src.idx = rows;
  src.rows1 = N;
  src.row_bytes = int4_row_bytes(K);
  src.num_groups = num_groups;
  LaunchOpts opts;
  opts.glu = as_half(glu_gate);
  cudaError_t e = launch_gemv_w4(RowMode::kIndexed, src, as_half(x), as_half(y), num_sel, K, group_size,
                                 as_stream(stream), opts);
  if (e == cudaErrorNotSupported && glu_gate) {  // shape outside the bulk path: GEMV, then the SwiGLU kernel
    e = launch_gemv_w4(RowMode::kIndexed, src, as_half(x), as_half(y), num_sel, K, group_size, as_stream(stream));
    if (e == cudaSuccess) e = launch_swiglu(as_half(glu_gate), as_half(y), rows, as_half(y), num_sel, as_stream(stream));
  }
  return cuda_result(e, name);
}

int soinfer_gemv_w8a16(const int8_t* Wq, const float* scale, const soinfer_half* x, soinfer_half* y, int64_t N,
                       int64_t K, int64_t group_size, int64_t num_groups, int64_t scale_row_stride, void* stream) {
  const char* name = "gemv_w8a16";
  REQUIRE(K >= 1 && N >= 0, "%s: invalid sizes", name);
  REQUIRE(group_size >= 1, "%s: group_size must be >= 1", name);
  REQUIRE(num_groups >= 1, "%s: num_groups must be >= 1", name);
  REQUIRE(num_groups == 1 || group_size % 4 == 0,
          "%s: group_size must be a multiple of 4 when num_groups > 1 (a 4-byte word never spans two groups)", name);
  REQUIRE(num_groups == 1 || num_groups == cdiv(K, group_size),
          "%s: scale's num_groups must be 1 (per-tensor broadcast) or ceil(K/group_size) for the given K and "
          "group_size, got %lld but expected %lld",
          name, (long long)num_groups, (long long)cdiv(K, group_size));
  REQUIRE(scale_row_stride == 0 || scale_row_stride == num_groups, "%s: scale_row_stride must be 0 or num_groups",
          name);
  if (N == 0) return SOINFER_OK;
  REQUIRE(Wq && scale && x && y, "%s: null pointer", name);
  return cuda_result(launch_gemv_w8(Wq, scale, as_half(x), as_half(y), N, K, group_size, num_groups,
                                    scale_row_stride, as_stream(stream)),
                     name);
}

static int topk_common(const char* name, bool exact, const float* v, int64_t n, int64_t k, int32_t* idx,
                       int32_t* count, void* stream) {
  REQUIRE(n >= 1 && n < (1ll << 31), "%s: abs_g must hold 1 .. 2^31-1 values", name);
  REQUIRE(k >= 1 && k <= n, "%s: k must be in [1, I]", name);
  REQUIRE(v && idx && count, "%s: null pointer", name);
  return cuda_result(launch_topk(exact, v, n, k, idx, count, as_stream(stream)), name);
}

int soinfer_topk_threshold_select(const float* abs_g, int64_t n, int64_t k, int32_t* out_idx, int32_t* out_count,
                                  void* stream) {
  return topk_common("topk_threshold_select", false, abs_g, n, k, out_idx, out_count, stream);
}

int soinfer_topk_threshold_select_abs_f16(const soinfer_half* gate, int64_t n, int64_t k, int32_t* out_idx,
                                          int32_t* out_count, void* stream) {
  const char* name = "topk_threshold_select_abs_f16";
  REQUIRE(n >= 1 && n < (1ll << 31), "%s: n must be in [1, 2^31)", name);
  REQUIRE(k >= 1 && k <= n, "%s: k must be in [1, n]", name);
  REQUIRE(gate && out_idx && out_count, "%s: null pointer", name);
  return cuda_result(launch_topk_abs_half(false, as_half(gate), n, k, out_idx, out_count, as_stream(stream)), name);
}

int soinfer_topk_select_exact(const float* abs_g, int64_t n, int64_t k, int32_t* out_idx, int32_t* out_count,
                              void* stream) {
  return topk_common("topk_select_exact", true, abs_g, n, k, out_idx, out_count, stream);
}

int soinfer_build_dip_descriptors(const int32_t* sel, int64_t k, const int32_t* slot_of, int64_t I, int32_t* desc,
                                  int32_t* miss, int32_t* miss_count, void* stream) {
  const char* name = "build_dip_descriptors";
  REQUIRE(k >= 0 && k < (1ll << 31) && I >= 0 && I < (1ll << 31), "%s: invalid sizes", name);
  REQUIRE(miss_count, "%s: null miss_count", name);
  REQUIRE(k == 0 || I >= 1, "%s: slot_of must be non-empty when channels are selected", name);
  REQUIRE(k == 0 || (sel && slot_of && desc && miss), "%s: null pointer", name);
  return cuda_result(launch_build_descriptors(sel, k, slot_of, I, desc, miss, miss_count, as_stream(stream)), name);
}

int soinfer_gemv_dip_fused_up(const uint8_t* cache_Wq, const float* cache_scale, int64_t C, const uint8_t* staging_Wq,
                              const float* staging_scale, int64_t M, const int32_t* desc, int64_t k,
                              const soinfer_half* x, soinfer_half* y, int64_t K, int64_t group_size,
                              int64_t num_groups, void* stream) {
  const char* name = "gemv_dip_fused_up";
  if (int st = check_int4_layout(name, K, group_size, num_groups)) return st;
  REQUIRE(C >= 0 && M >= 0 && k >= 0, "%s: sizes must be >= 0", name);
  if (k == 0) return SOINFER_OK;
  REQUIRE(C + M >= 1, "%s: descriptors given but both cache and staging are empty", name);
  REQUIRE(desc && x && y, "%s: null pointer", name);
  REQUIRE((C == 0 || (cache_Wq && cache_scale)) && (M == 0 || (staging_Wq && staging_scale)), "%s: null row buffer",
          name);
  RowSource src;
  src.W = cache_Wq;
  src.S = cache_scale;
  src.W2 = staging_Wq;
  src.S2 = staging_scale;
  src.idx = desc;
  src.rows1 = C;
  src.rows2 = M;
  src.row_bytes = int4_row_bytes(K);
  src.num_groups = num_groups;
  return cuda_result(launch_gemv_w4(RowMode::kDesc, src, as_half(x), as_half(y), k, K, group_size, as_stream(stream)),
                     name);
}

int soinfer_gemv_fp16(const soinfer_half* W, const soinfer_half* x, soinfer_half* y, int64_t N, int64_t K,
                      void* stream) {
  const char* name = "gemv_fp16_v3";
  REQUIRE(N >= 0 && K >= 1, "%s: N must be >= 0 and K >= 1", name);
  REQUIRE(K % 8 == 0, "%s: K must be a multiple of 8 (float4-vectorized loads)", name);
  if (N == 0) return SOINFER_OK;
  REQUIRE(W && x && y, "%s: null pointer", name);
  REQUIRE(aligned(W, 16) && aligned(x, 16) && aligned(y, 2), "%s: W and x must be 16-byte aligned", name);
  return cuda_result(launch_gemv_fp16(as_half(W), as_half(x), as_half(y), N, K, as_stream(stream)), name);
}

int64_t soinfer_lm_head_argmax_workspace_bytes(void) { return lm_head_argmax_workspace_bytes(); }

int soinfer_gemv_fp16_argmax(const soinfer_half* W, const soinfer_half* x, soinfer_half* y, int64_t N, int64_t K,
                             int32_t* out_idx, void* workspace, int64_t workspace_bytes, void* stream) {
  const char* name = "gemv_fp16_argmax";
  REQUIRE(N >= 1 && N < (int64_t)1 << 31 && K >= 1, "%s: N must be in [1, 2^31) and K >= 1", name);
  REQUIRE(K % 8 == 0, "%s: K must be a multiple of 8 (float4-vectorized loads)", name);
  REQUIRE(W && x && out_idx, "%s: null pointer", name);
  REQUIRE(aligned(W, 16) && aligned(x, 16) && aligned(y, 2), "%s: W and x must be 16-byte aligned", name);
  REQUIRE(workspace && workspace_bytes >= lm_head_argmax_workspace_bytes() && aligned(workspace, 8),
          "%s: workspace too small (need %lld zeroed bytes)", name, (long long)lm_head_argmax_workspace_bytes());
  return cuda_result(launch_gemv_fp16_argmax(as_half(W), as_half(x), as_half(y), N, K, workspace, out_idx,
                                             as_stream(stream)),
                     name);
}

int64_t soinfer_sparse_workspace_bytes(int64_t H, int64_t k) {
  if (H < 1 || k < 0) return 0;
  return sparse_workspace_bytes(H, k > 0 ? k : 1);
}

static int sparse_common(const char* name, RowMode mode, const RowSource& src, const soinfer_half* h, soinfer_half* y,
                         int64_t H, int64_t k, int64_t group_size, int64_t num_groups, void* ws, int64_t ws_bytes,
                         void* stream, const soinfer_half* residual = nullptr) {
  if (int st = check_int4_layout(name, H, group_size, num_groups)) return st;
  REQUIRE(k >= 0, "%s: k must be >= 0", name);
  REQUIRE(y, "%s: null output", name);
  if (k == 0) {
    if (residual) return cuda_result(cudaMemcpyAsync(y, residual, (size_t)H * 2, cudaMemcpyDeviceToDevice,
                                                     as_stream(stream)), name);
    return cuda_result(cudaMemsetAsync(y, 0, (size_t)H * 2, as_stream(stream)), name);
  }
  REQUIRE(h, "%s: null h", name);
  REQUIRE(ws && ws_bytes >= sparse_workspace_bytes(H, k), "%s: workspace too small (need %lld bytes)", name,
          (long long)sparse_workspace_bytes(H, k));
  REQUIRE(aligned(ws, 16), "%s: workspace must be 16-byte aligned", name);
  LaunchOpts opts;
  opts.resid = as_half(residual);
  return cuda_result(
      launch_sparse_down(mode, src, as_half(h), as_half(y), H, k, group_size, ws, as_stream(stream), opts), name);
}

int soinfer_gemv_w4a16_sparse_accumulate(const uint8_t* Wq_sel, const float* scale_sel, const soinfer_half* h,
                                         soinfer_half* y, int64_t H, int64_t k, int64_t group_size, int64_t num_groups,
                                         void* workspace, int64_t workspace_bytes, void* stream) {
  const char* name = "gemv_w4a16_sparse_accumulate";
  REQUIRE(k == 0 || (Wq_sel && scale_sel), "%s: null pointer", name);
  REQUIRE(aligned(Wq_sel, 4), "%s: misaligned weights", name);
  RowSource src;
  src.W = Wq_sel;
  src.S = scale_sel;
  src.rows1 = k;
  src.row_bytes = int4_row_bytes(H);
  src.num_groups = num_groups;
  return sparse_common(name, RowMode::kPlain, src, h, y, H, k, group_size, num_groups, workspace, workspace_bytes,
                       stream);
}

int soinfer_gemv_w4a16_sparse_accumulate_noalloc(const uint8_t* Wq_sel, const float* scale_sel, const soinfer_half* h,
                                                 soinfer_half* y, int64_t H, int64_t k, int64_t group_size,
                                                 int64_t num_groups, void* stream) {
  const char* name = "gemv_w4a16_sparse_accumulate_noalloc";
  REQUIRE(k == 0 || (Wq_sel && scale_sel), "%s: null pointer", name);
  REQUIRE(aligned(Wq_sel, 4), "%s: misaligned weights", name);
  if (int st = check_int4_layout(name, H, group_size, num_groups)) return st;
  REQUIRE(k >= 0, "%s: k must be >= 0", name);
  REQUIRE(y, "%s: null output", name);
  if (k == 0) return cuda_result(cudaMemsetAsync(y, 0, (size_t)H * 2, as_stream(stream)), name);
  REQUIRE(h, "%s: null h", name);
  REQUIRE(sparse_workspace_bytes(H, k) <= sparse_static_scratch_bytes(),
          "%s: H=%lld, k=%lld needs %lld scratch bytes, above the static %lld", name, (long long)H, (long long)k,
          (long long)sparse_workspace_bytes(H, k), (long long)sparse_static_scratch_bytes());
  void* scratch = nullptr;
  if (int st = cuda_result(sparse_static_scratch(&scratch, as_stream(stream)), name)) return st;
  RowSource src;
  src.W = Wq_sel;
  src.S = scale_sel;
  src.rows1 = k;
  src.row_bytes = int4_row_bytes(H);
  src.num_groups = num_groups;
  return cuda_result(launch_sparse_down(RowMode::kPlain, src, as_half(h), as_half(y), H, k, group_size, scratch,
                                        as_stream(stream)),
                     name);
}

int soinfer_gemv_w4a16_sparse_rows(const uint8_t* Wq_T, const float* scale_T, int64_t I, const int32_t* rows,
                                   const soinfer_half* h, soinfer_half* y, int64_t H, int64_t k, int64_t group_size,
                                   int64_t num_groups, void* workspace, int64_t workspace_bytes,
                                   const soinfer_half* residual, void* stream) {
  const char* name = "gemv_w4a16_sparse_rows";
  REQUIRE(k == 0 || (I >= 1 && Wq_T && scale_T && rows), "%s: null pointer or empty matrix", name);
  REQUIRE(aligned(Wq_T, 4), "%s: misaligned weights", name);
  RowSource src;
  src.W = Wq_T;
  src.S = scale_T;
  src.idx = rows;
  src.rows1 = I;
  src.row_bytes = int4_row_bytes(H);
  src.num_groups = num_groups;
  return sparse_common(name, RowMode::kIndexed, src, h, y, H, k, group_size, num_groups, workspace, workspace_bytes,
                       stream, residual);
}

int soinfer_gemv_dip_fused_down(const uint8_t* cache_Wq, const float* cache_scale, int64_t C,
                                const uint8_t* staging_Wq, const float* staging_scale, int64_t M, const int32_t* desc,
                                const soinfer_half* h, soinfer_half* y, int64_t H, int64_t k, int64_t group_size,
                                int64_t num_groups, void* workspace, int64_t workspace_bytes, void* stream) {
  const char* name = "gemv_dip_fused_down";
  REQUIRE(C >= 0 && M >= 0, "%s: sizes must be >= 0", name);
  REQUIRE(k == 0 || (C + M >= 1 && desc), "%s: descriptors given but both cache and staging are empty", name);
  REQUIRE((C == 0 || (cache_Wq && cache_scale)) && (M == 0 || (staging_Wq && staging_scale)), "%s: null row buffer",
          name);
  REQUIRE(aligned(cache_Wq, 4) && aligned(staging_Wq, 4), "%s: misaligned weights", name);
  RowSource src;
  src.W = cache_Wq;
  src.S = cache_scale;
  src.W2 = staging_Wq;
  src.S2 = staging_scale;
  src.idx = desc;
  src.rows1 = C;
  src.rows2 = M;
  src.row_bytes = int4_row_bytes(H);
  src.num_groups = num_groups;
  return sparse_common(name, RowMode::kDesc, src, h, y, H, k, group_size, num_groups, workspace, workspace_bytes,
                       stream);
}

int soinfer_gather_rows_device(const uint8_t* matrix, int64_t num_rows, int64_t row_nbytes, const int32_t* rows,
                               int64_t k, uint8_t* gpu_dst, void* stream) {
  const char* name = "gather_rows_device";
  REQUIRE(num_rows >= 0 && row_nbytes >= 0 && k >= 0, "%s: sizes must be >= 0", name);
  if (k == 0 || row_nbytes == 0) return SOINFER_OK;
  REQUIRE(num_rows >= 1 && matrix && rows && gpu_dst, "%s: null pointer or empty matrix", name);
  return cuda_result(launch_gather_rows_device(matrix, num_rows, row_nbytes, rows, k, gpu_dst, as_stream(stream)),
                     name);
}

int soinfer_gather_rows_device_multi(const soinfer_gather_src* srcs, int32_t num_srcs, const int32_t* rows,
                                     const int32_t* count, int64_t max_k, void* stream) {
  const char* name = "gather_rows_device_multi";
  REQUIRE(num_srcs >= 0 && num_srcs <= kMaxGatherSrc, "%s: num_srcs must be in [0, %d]", name, kMaxGatherSrc);
  REQUIRE(max_k >= 0, "%s: max_k must be >= 0", name);
  if (num_srcs == 0 || max_k == 0) return SOINFER_OK;
  REQUIRE(srcs && rows, "%s: null pointer", name);
  GatherMulti P = {};
  P.num = num_srcs;
  P.rows = rows;
  P.count = count;
  P.max_k = max_k;
  for (int i = 0; i < num_srcs; ++i) {
    const soinfer_gather_src& g = srcs[i];
    REQUIRE(g.matrix && g.dst && g.num_rows >= 1, "%s: source %d: null pointer or empty matrix", name, i);
    REQUIRE(g.row_nbytes >= 4 && g.row_nbytes % 4 == 0 && aligned(g.matrix, 4) && aligned(g.dst, 4),
            "%s: source %d: row_nbytes must be a positive multiple of 4 with 4-byte aligned matrix / dst", name, i);
    P.src[i] = GatherSrc{g.matrix, g.num_rows, g.row_nbytes, g.dst,
                         (g.row_nbytes % 16 == 0 && aligned(g.matrix, 16) && aligned(g.dst, 16)) ? 1 : 0};
  }
  return cuda_result(launch_gather_multi(P, as_stream(stream)), name);
}

int soinfer_rmsnorm(const soinfer_half* x, const soinfer_half* weight, soinfer_half* out, int64_t rows, int64_t hidden,
                    float eps, void* stream) {
  const char* name = "rmsnorm";
  REQUIRE(rows >= 0 && rows < (1ll << 31), "%s: invalid rows", name);
  REQUIRE(hidden >= 2 && hidden % 2 == 0, "%s: hidden dim must be even (half2 vectorization)", name);
  if (rows == 0) return SOINFER_OK;
  REQUIRE(x && weight && out, "%s: null pointer", name);
  REQUIRE(aligned(x, 4) && aligned(weight, 4) && aligned(out, 4), "%s: misaligned pointer", name);
  return cuda_result(launch_rmsnorm(as_half(x), as_half(weight), as_half(out), rows, hidden, eps, as_stream(stream)),
                     name);
}

int soinfer_rope_apply(soinfer_half* x, const float* cos_vals, const float* sin_vals, int64_t num_heads,
                       int64_t head_dim, void* stream) {
  const char* name = "rope_apply";
  REQUIRE(num_heads >= 0 && num_heads < (1ll << 31), "%s: invalid num_heads", name);
  REQUIRE(head_dim >= 2 && head_dim % 2 == 0, "%s: head_dim must be even", name);
  if (num_heads == 0) return SOINFER_OK;
  REQUIRE(x && cos_vals && sin_vals, "%s: null pointer", name);
  return cuda_result(launch_rope(as_half(x), cos_vals, sin_vals, num_heads, head_dim, as_stream(stream)), name);
}

int soinfer_kv_cache_append(soinfer_half* k_cache, soinfer_half* v_cache, const soinfer_half* k_new,
                            const soinfer_half* v_new, int64_t num_kv_heads, int64_t max_seq_len, int64_t head_dim,
                            int64_t pos, void* stream) {
  const char* name = "kv_cache_append";
  REQUIRE(num_kv_heads >= 0 && max_seq_len >= 1 && head_dim >= 1, "%s: invalid cache shape", name);
  REQUIRE(pos >= 0 && pos < max_seq_len, "%s: pos out of range for max_seq_len", name);
  if (num_kv_heads == 0) return SOINFER_OK;
  REQUIRE(k_cache && v_cache && k_new && v_new, "%s: null pointer", name);
  return cuda_result(launch_kv_append(as_half(k_cache), as_half(v_cache), as_half(k_new), as_half(v_new), num_kv_heads,
                                      max_seq_len, head_dim, pos, as_stream(stream)),
                     name);
}

int64_t soinfer_decode_attention_workspace_bytes(int64_t num_q_heads, int64_t max_seq_len, int64_t head_dim) {
  if (num_q_heads < 1 || head_dim < 1) return 0;
  return attention_workspace_bytes(num_q_heads, max_seq_len, head_dim);
}

int soinfer_decode_attention(const soinfer_half* q, const soinfer_half* k_cache, const soinfer_half* v_cache,
                             soinfer_half* out, int64_t num_q_heads, int64_t num_kv_heads, int64_t max_seq_len,
                             int64_t head_dim, int64_t cur_len, void* workspace, int64_t workspace_bytes,
                             void* stream) {
  const char* name = "decode_attention";
  REQUIRE(num_kv_heads >= 1 && num_q_heads >= 1, "%s: head counts must be >= 1", name);
  REQUIRE(num_q_heads % num_kv_heads == 0, "%s: num_q_heads must be a multiple of num_kv_heads", name);
  REQUIRE(head_dim >= 8 && head_dim % 8 == 0 && head_dim <= 256, "%s: head_dim must be a multiple of 8 in [8, 256]",
          name);
  REQUIRE(cur_len >= 1 && cur_len <= max_seq_len, "%s: cur_len out of range for max_seq_len", name);
  REQUIRE(num_q_heads <= 1024 && max_seq_len < (1ll << 31), "%s: sizes too large (num_q_heads <= 1024)", name);
  REQUIRE(q && k_cache && v_cache && out, "%s: null pointer", name);
  REQUIRE(aligned(q, 16) && aligned(k_cache, 16) && aligned(v_cache, 16), "%s: q and caches must be 16-byte aligned",
          name);
  REQUIRE(workspace && workspace_bytes >= attention_workspace_bytes(num_q_heads, max_seq_len, head_dim),
          "%s: workspace too small", name);
  return cuda_result(launch_decode_attention(as_half(q), as_half(k_cache), as_half(v_cache), as_half(out), num_q_heads,
                                             num_kv_heads, max_seq_len, head_dim, cur_len, workspace,
                                             as_stream(stream)),
                     name);
}

int soinfer_add_rmsnorm(const soinfer_half* x, const soinfer_half* x2, const soinfer_half* weight, soinfer_half* out,
                        soinfer_half* sum_out, int64_t rows, int64_t hidden, float eps, void* stream) {
  const char* name = "add_rmsnorm";
  REQUIRE(rows >= 0 && rows < (1ll << 31) && hidden >= 2 && hidden % 2 == 0, "%s: invalid shape (hidden even)", name);
  if (rows == 0) return SOINFER_OK;
  REQUIRE(x && x2 && weight && out && sum_out, "%s: null pointer", name);
  REQUIRE(aligned(x, 4) && aligned(x2, 4) && aligned(weight, 4) && aligned(out, 4) && aligned(sum_out, 4),
          "%s: misaligned pointer", name);
  return cuda_result(launch_add_rmsnorm(as_half(x), as_half(x2), as_half(weight), as_half(out), as_half(sum_out), rows,
                                        hidden, eps, as_stream(stream)),
                     name);
}

int soinfer_swiglu(const soinfer_half* gate, const soinfer_half* up, const int32_t* idx, soinfer_half* out, int64_t n,
                   void* stream) {
  const char* name = "swiglu";
  REQUIRE(n >= 0, "%s: n must be >= 0", name);
  if (n == 0) return SOINFER_OK;
  REQUIRE(gate && up && out, "%s: null pointer", name);
  return cuda_result(launch_swiglu(as_half(gate), as_half(up), idx, as_half(out), n, as_stream(stream)), name);
}

int soinfer_head_norm_rope(soinfer_half* q, const soinfer_half* k, const soinfer_half* v, const soinfer_half* q_norm,
                           const soinfer_half* k_norm, const float* cos_vals, const float* sin_vals, int64_t table_rows,
                           soinfer_half* k_cache, soinfer_half* v_cache, int64_t num_q_heads, int64_t num_kv_heads,
                           int64_t head_dim, int64_t max_seq_len, int64_t pos, const int32_t* pos_dev, float eps,
                           void* stream) {
  const char* name = "head_norm_rope";
  REQUIRE(num_q_heads >= 1 && num_kv_heads >= 1 && num_q_heads + 2 * num_kv_heads < (1ll << 30),
          "%s: invalid head counts", name);
  REQUIRE(head_dim >= 2 && head_dim % 2 == 0 && head_dim <= 256, "%s: head_dim must be even and <= 256", name);
  REQUIRE(max_seq_len >= 1, "%s: invalid max_seq_len", name);
  REQUIRE(pos_dev || (pos >= 0 && pos < max_seq_len), "%s: pos out of range for max_seq_len", name);
  REQUIRE(!pos_dev || table_rows >= 1, "%s: table_rows must be >= 1 with pos_dev", name);
  REQUIRE(q && k && v && q_norm && k_norm && cos_vals && sin_vals && k_cache && v_cache, "%s: null pointer", name);
  return cuda_result(launch_head_norm_rope(as_half(q), as_half(k), as_half(v), as_half(q_norm), as_half(k_norm),
                                           cos_vals, sin_vals, as_half(k_cache), as_half(v_cache), num_q_heads,
                                           num_kv_heads, head_dim, max_seq_len, pos, pos_dev, table_rows, eps,
                                           as_stream(stream)),
                     name);
}

int soinfer_rope_apply_at(soinfer_half* x, const float* cos_table, const float* sin_table, int64_t table_rows,
                          int64_t num_heads, int64_t head_dim, const int32_t* pos_dev, void* stream) {
  const char* name = "rope_apply_at";
  REQUIRE(num_heads >= 0 && num_heads < (1ll << 31) && table_rows >= 1, "%s: invalid num_heads / table_rows", name);
  REQUIRE(head_dim >= 2 && head_dim % 2 == 0, "%s: head_dim must be even", name);
  if (num_heads == 0) return SOINFER_OK;
  REQUIRE(x && cos_table && sin_table && pos_dev, "%s: null pointer", name);
  return cuda_result(launch_rope_at(as_half(x), cos_table, sin_table, table_rows, num_heads, head_dim, pos_dev,
                                    as_stream(stream)),
                     name);
}

int soinfer_kv_cache_append_at(soinfer_half* k_cache, soinfer_half* v_cache, const soinfer_half* k_new,
                               const soinfer_half* v_new, int64_t num_kv_heads, int64_t max_seq_len, int64_t head_dim,
                               const int32_t* pos_dev, void* stream) {
  const char* name = "kv_cache_append_at";
  REQUIRE(num_kv_heads >= 0 && max_seq_len >= 1 && head_dim >= 1, "%s: invalid cache shape", name);
  if (num_kv_heads == 0) return SOINFER_OK;
  REQUIRE(k_cache && v_cache && k_new && v_new && pos_dev, "%s: null pointer", name);
  return cuda_result(launch_kv_append_at(as_half(k_cache), as_half(v_cache), as_half(k_new), as_half(v_new),
                                         num_kv_heads, max_seq_len, head_dim, pos_dev, as_stream(stream)),
                     name);
}

int soinfer_decode_attention_at(const soinfer_half* q, const soinfer_half* k_cache, const soinfer_half* v_cache,
                                soinfer_half* out, int64_t num_q_heads, int64_t num_kv_heads, int64_t max_seq_len,
                                int64_t head_dim, const int32_t* pos_dev, void* workspace, int64_t workspace_bytes,
                                void* stream) {
  const char* name = "decode_attention_at";
  REQUIRE(num_kv_heads >= 1 && num_q_heads >= 1, "%s: head counts must be >= 1", name);
  REQUIRE(num_q_heads % num_kv_heads == 0, "%s: num_q_heads must be a multiple of num_kv_heads", name);
  REQUIRE(head_dim >= 8 && head_dim % 8 == 0 && head_dim <= 256, "%s: head_dim must be a multiple of 8 in [8, 256]",
          name);
  REQUIRE(max_seq_len >= 1 && num_q_heads <= 1024 && max_seq_len < (1ll << 31), "%s: sizes out of range (num_q_heads <= 1024)", name);
  REQUIRE(q && k_cache && v_cache && out && pos_dev, "%s: null pointer", name);
  REQUIRE(aligned(q, 16) && aligned(k_cache, 16) && aligned(v_cache, 16), "%s: q and caches must be 16-byte aligned",
          name);
  REQUIRE(workspace && workspace_bytes >= attention_workspace_bytes(num_q_heads, max_seq_len, head_dim),
          "%s: workspace too small", name);
  return cuda_result(launch_decode_attention_at(as_half(q), as_half(k_cache), as_half(v_cache), as_half(out),
                                                num_q_heads, num_kv_heads, max_seq_len, head_dim, pos_dev, workspace,
                                                as_stream(stream)),
                     name);
}

int soinfer_decode_step_embed(const soinfer_half* embed, int64_t vocab, int64_t hidden, const int32_t* ids,
                              int64_t ids_len, const int32_t* pos_dev, soinfer_half* x, void* stream) {
  const char* name = "decode_step_embed";
  REQUIRE(vocab >= 1 && hidden >= 1 && ids_len >= 1 && hidden < (1ll << 31), "%s: invalid sizes", name);
  REQUIRE(embed && ids && pos_dev && x, "%s: null pointer", name);
  return cuda_result(launch_step_embed(as_half(embed), vocab, hidden, ids, ids_len, pos_dev, as_half(x),
                                       as_stream(stream)),
                     name);
}

int soinfer_decode_step_advance(int32_t* ids, int64_t ids_len, int32_t* pos_dev, const int32_t* prompt_len,
                                const int32_t* next, void* stream) {
  const char* name = "decode_step_advance";
  REQUIRE(ids_len >= 1, "%s: ids_len must be >= 1", name);
  REQUIRE(ids && pos_dev && prompt_len && next, "%s: null pointer", name);
  return cuda_result(launch_step_advance(ids, ids_len, pos_dev, prompt_len, next, as_stream(stream)), name);
}

int soinfer_gemm_w4a16(const uint8_t* Wq, const float* scale, const soinfer_half* X, int64_t ldx, soinfer_half* Y,
                       int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group_size, int64_t num_groups,
                       void* stream) {
  const char* name = "gemm_w4a16";
  if (int st = check_int4_layout(name, K, group_size, num_groups)) return st;
  REQUIRE(M >= 0 && M <= 8, "%s: M (tokens) must be in [0, 8]", name);
  REQUIRE(N >= 0, "%s: N must be >= 0", name);
  if (M == 0 || N == 0) return SOINFER_OK;
  REQUIRE(Wq && scale && X && Y, "%s: null pointer", name);
  REQUIRE(ldx >= K && ldy >= N, "%s: row strides must cover K / N", name);
  REQUIRE(aligned(Wq, 4) && aligned(scale, 4) && aligned(X, 2) && aligned(Y, 2), "%s: misaligned pointer", name);
  cudaStream_t st = as_stream(stream);
  const bool fast = plan_gemm_w4(M, N, K, group_size, num_groups) && aligned(Wq, 16) && aligned(scale, 16) &&
                    aligned(X, 16) && ldx % 8 == 0;
  if (fast) {
    const cudaError_t e = launch_gemm_w4(Wq, scale, as_half(X), ldx, as_half(Y), ldy, M, N, K, group_size,
                                         num_groups, st);
    if (e != cudaErrorNotSupported) return cuda_result(e, name);
  }
  // per-token fallback: the single-token GEMV on each row of X
  RowSource src;
  src.W = Wq;
  src.S = scale;
  src.rows1 = N;
  src.row_bytes = int4_row_bytes(K);
  src.num_groups = num_groups;
  for (int64_t m = 0; m < M; ++m)
    if (int rc = cuda_result(launch_gemv_w4(RowMode::kPlain, src, as_half(X) + m * ldx, as_half(Y) + m * ldy, N, K,
                                            group_size, st),
                             name))
      return rc;
  return SOINFER_OK;
}

int soinfer_quantize_pack_int4(const void* w, int32_t dtype, int64_t N, int64_t K, int64_t ld, int64_t group_size,
                               uint8_t* packed, float* scale, void* stream) {
  const char* name = "quantize_pack_int4";
  REQUIRE(dtype >= 0 && dtype <= 2, "%s: dtype must be 0 (fp32), 1 (fp16) or 2 (bf16)", name);
  REQUIRE(group_size >= 8 && group_size <= 256 && (group_size & (group_size - 1)) == 0,
          "%s: group_size must be a power of two in [8, 256]", name);
  REQUIRE(N >= 0 && K >= 1 && ld >= K && N < (1ll << 40) && K < (1ll << 31), "%s: invalid shape or row stride", name);
  if (N == 0) return SOINFER_OK;
  REQUIRE(w && packed && scale, "%s: null pointer", name);
  REQUIRE(aligned(packed, 4) && aligned(scale, 4), "%s: packed and scale must be 4-byte aligned", name);
  return cuda_result(launch_quantize_pack_int4(w, dtype, N, K, ld, group_size, packed, scale, as_stream(stream)),
                     name);
}

// ---------------------------------------------------------------- tensor-parallel exchange

static_assert(sizeof(cudaIpcMemHandle_t) == SOINFER_IPC_HANDLE_BYTES, "IPC handle size");
static_assert(SOINFER_MAX_PEERS == kMaxPeers, "peer count");

namespace {
int to_peer_set(const char* name, const soinfer_peer_set* in, PeerSet& ps) {
  REQUIRE(in, "%s: null peer set", name);
  REQUIRE(in->world >= 1 && in->world <= kMaxPeers, "%s: world size must be in [1, %d]", name, kMaxPeers);
  REQUIRE(in->rank >= 0 && in->rank < in->world, "%s: rank out of range", name);
  REQUIRE(in->slot_bytes >= 16 && in->slot_bytes % 16 == 0 && in->slot_bytes < (1ll << 31),
          "%s: slot_bytes must be a positive multiple of 16", name);
  for (int r = 0; r < kMaxPeers; ++r) {
    if (r < in->world) {
      REQUIRE(in->base[r] && aligned(in->base[r], 256), "%s: peer buffer %d null or not 256-byte aligned", name, r);
    }
    ps.base[r] = r < in->world ? static_cast<uint8_t*>(in->base[r]) : nullptr;
  }
  ps.rank = in->rank;
  ps.world = in->world;
  ps.slot_bytes = in->slot_bytes;
  return SOINFER_OK;
}
}  // namespace

int64_t soinfer_peer_buffer_bytes(int64_t slot_bytes, int32_t world) {
  if (slot_bytes < 16 || slot_bytes % 16 || world < 1 || world > kMaxPeers) return 0;
  return peer_buffer_bytes(slot_bytes, world);
}

int soinfer_peer_buffer_create(int64_t bytes, void** dptr, void* ipc_handle) {
  const char* name = "peer_buffer_create";
  REQUIRE(dptr && ipc_handle, "%s: null output pointer", name);
  REQUIRE(bytes >= kPeerHeaderBytes, "%s: buffer smaller than its header", name);
  *dptr = nullptr;
  void* p = nullptr;
  if (int st = cuda_result(cudaMalloc(&p, (size_t)bytes), name)) return st;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaMemset(p, 0, (size_t)bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // zeroed before any stream (blocking or not) uses it
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_result(e, name);
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *dptr = p;
  return SOINFER_OK;
}

int soinfer_peer_buffer_open(const void* ipc_handle, void** dptr) {
  const char* name = "peer_buffer_open";
  REQUIRE(ipc_handle && dptr, "%s: null pointer", name);
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  *dptr = nullptr;
  return cuda_result(cudaIpcOpenMemHandle(dptr, h, cudaIpcMemLazyEnablePeerAccess), name);
}

int soinfer_peer_buffer_close(void* dptr) {
  REQUIRE(dptr, "peer_buffer_close: null pointer");
  return cuda_result(cudaIpcCloseMemHandle(dptr), "peer_buffer_close");
}

int soinfer_peer_buffer_destroy(void* dptr) {
  REQUIRE(dptr, "peer_buffer_destroy: null pointer");
  return cuda_result(cudaFree(dptr), "peer_buffer_destroy");
}

int soinfer_peer_buffer_reset(void* dptr, void* stream) {
  REQUIRE(dptr, "peer_buffer_reset: null pointer");
  return cuda_result(cudaMemsetAsync(dptr, 0, (size_t)kPeerHeaderBytes, as_stream(stream)), "peer_buffer_reset");
}

int soinfer_tp_allreduce_add_rmsnorm(const soinfer_peer_set* peers, const soinfer_half* partial,
                                     const soinfer_half* residual, const soinfer_half* weight, soinfer_half* out_sum,
                                     soinfer_half* out_norm, int64_t n, float eps, void* stream) {
  const char* name = "tp_allreduce_add_rmsnorm";
  PeerSet ps;
  if (int st = to_peer_set(name, peers, ps)) return st;
  REQUIRE(n >= 8 && n % 8 == 0 && n * 2 <= ps.slot_bytes, "%s: n must be a multiple of 8 with 2n <= slot_bytes",
          name);
  REQUIRE(out_sum && (!out_norm || weight), "%s: null output (or weight with out_norm)", name);
  REQUIRE(aligned(out_sum, 16) && aligned(partial, 16) && aligned(residual, 16) && aligned(weight, 16) &&
              aligned(out_norm, 16),
          "%s: vectors must be 16-byte aligned", name);
  return cuda_result(launch_tp_allreduce_norm(ps, as_half(partial), as_half(residual), as_half(weight),
                                              as_half(out_sum), as_half(out_norm), n, eps, as_stream(stream)),
                     name);
}

int soinfer_gemv_w4a16_tp_partial(const soinfer_peer_set* peers, const uint8_t* Wq, const float* scale,
                                  const soinfer_half* x, int64_t N, int64_t K, int64_t group_size, int64_t num_groups,
                                  void* stream) {
  const char* name = "gemv_w4a16_tp_partial";
  PeerSet ps;
  if (int st = to_peer_set(name, peers, ps)) return st;
  if (int st = check_int4_layout(name, K, group_size, num_groups)) return st;
  REQUIRE(N >= 1 && N * 2 <= ps.slot_bytes, "%s: N must be >= 1 with 2N <= slot_bytes", name);
  REQUIRE(K % 128 == 0 && group_size % 128 == 0, "%s: K and group_size must be multiples of 128", name);
  REQUIRE(Wq && scale && x, "%s: null pointer", name);
  REQUIRE(aligned(Wq, 16) && aligned(scale, 16) && aligned(x, 16), "%s: Wq, scale and x must be 16-byte aligned",
          name);
  RowSource src;
  src.W = Wq;
  src.S = scale;
  src.rows1 = N;
  src.row_bytes = int4_row_bytes(K);
  src.num_groups = num_groups;
  const cudaError_t e = launch_gemv_w4_peer(src, as_half(x), N, K, group_size, ps, as_stream(stream));
  if (e == cudaErrorNotSupported)
    return set_error(SOINFER_ERR_UNSUPPORTED, "%s: shape outside the bulk GEMV path (rows too wide for one CTA)", name);
  return cuda_result(e, name);
}

int soinfer_gemv_w4a16_batch_tp(const soinfer_peer_set* peers, const soinfer_gemv_task* tasks, int64_t num_tasks,
                                void* workspace, int64_t workspace_bytes, void* stream) {
  const char* name = "gemv_w4a16_batch_tp";
  PeerSet ps;
  if (int st = to_peer_set(name, peers, ps)) return st;
  return gemv_batch_common(name, &ps, tasks, num_tasks, workspace, workspace_bytes, stream);
}

int soinfer_tp_allgather(const soinfer_peer_set* peers, const void* local, int64_t nbytes, void* out, void* stream) {
  const char* name = "tp_allgather";
  PeerSet ps;
  if (int st = to_peer_set(name, peers, ps)) return st;
  REQUIRE(nbytes >= 16 && nbytes % 16 == 0 && nbytes <= ps.slot_bytes,
          "%s: nbytes must be a positive multiple of 16, at most slot_bytes", name);
  REQUIRE(local && out && aligned(local, 16) && aligned(out, 16), "%s: null or misaligned buffer", name);
  return cuda_result(launch_tp_allgather(ps, local, nbytes, out, as_stream(stream)), name);
}

int soinfer_tp_argmax(const soinfer_peer_set* peers, const soinfer_half* logits, const int32_t* local_idx,
                      int64_t offset, int32_t* out_idx, void* stream) {
  const char* name = "tp_argmax";
  PeerSet ps;
  if (int st = to_peer_set(name, peers, ps)) return st;
  REQUIRE(ps.slot_bytes >= 16, "%s: slot too small", name);
  REQUIRE(logits && local_idx && out_idx, "%s: null pointer", name);
  REQUIRE(offset >= 0 && offset < (1ll << 31), "%s: offset out of range", name);
  return cuda_result(launch_tp_argmax(ps, as_half(logits), local_idx, offset, out_idx, as_stream(stream)), name);
}

}  // extern "C"
