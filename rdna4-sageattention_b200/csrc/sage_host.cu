// sage_attention_host: the whole attention call on tensors in host memory.  The heads are cut into
// chunks (whole groups of query heads sharing a kv head); chunk c is copied in on one stream, attended
// on the caller's stream (even c) or a second compute stream (odd c) and copied out on a fourth, so the
// host<->device copies of neighbouring chunks overlap the kernels of the current one, and the CTAs of
// chunk c+1 fill the SMs that the last wave of chunk c leaves idle.  Device staging and quantised-tensor
// scratch for two chunks in flight are carved from the caller's workspace; the library allocates
// nothing.
#include <algorithm>
#include <cmath>
#include <mutex>
#include <vector>

#include "../../include/sage_b200.h"
#include "sage_internal.h"

namespace sage {
namespace {

constexpr int kMaxDevices = 64;

// Per-device copy streams, the compute stream of odd chunks and the events that order the two staging
// slots.
struct HostPipe {
  bool ready = false;
  cudaStream_t in = nullptr, out = nullptr, comp = nullptr;
  cudaEvent_t start = nullptr;
  cudaEvent_t in_done[2] = {nullptr, nullptr};
  cudaEvent_t comp_done[2] = {nullptr, nullptr};
  cudaEvent_t out_done[2] = {nullptr, nullptr};
};

std::mutex g_pipe_mu;
HostPipe g_pipe[kMaxDevices];

// Called with g_pipe_mu held.
HostPipe* pipe_for_current_device(int* dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  *dev_out = dev;
  HostPipe& p = g_pipe[dev];
  if (p.ready) return &p;
  bool ok = cudaStreamCreateWithFlags(&p.in, cudaStreamNonBlocking) == cudaSuccess &&
            cudaStreamCreateWithFlags(&p.out, cudaStreamNonBlocking) == cudaSuccess &&
            cudaStreamCreateWithFlags(&p.comp, cudaStreamNonBlocking) == cudaSuccess &&
            cudaEventCreateWithFlags(&p.start, cudaEventDisableTiming) == cudaSuccess;
  for (int i = 0; ok && i < 2; ++i)
    ok = cudaEventCreateWithFlags(&p.in_done[i], cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&p.comp_done[i], cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&p.out_done[i], cudaEventDisableTiming) == cudaSuccess;
  if (!ok) return nullptr;
  p.ready = true;
  return &p;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Layout of one tensor's chunk on the device: token-major (B, S, hg, D) when the host tensor keeps a
// token's heads next to each other (head stride == D, e.g. NHD), so each batch is one pitched copy;
// head-major (B, hg, S, D) otherwise (HND and other layouts).
struct ChunkLayout {
  bool token_major;
  Strides3 st;  // element strides of the device chunk
};

ChunkLayout chunk_layout(const Strides3& host, int S, int hg, int D) {
  if (host.h == D) return {true, Strides3{(int64_t)S * hg * D, (int64_t)hg * D, D}};
  return {false, Strides3{(int64_t)hg * S * D, D, (int64_t)S * D}};
}

// Copies heads [h0, h0 + hg) of a (B, S, H, D) tensor with host strides `hs` to (to_dev) or from the
// device chunk `dev` laid out as `L`, with one cudaMemcpyAsync / cudaMemcpy2DAsync per contiguous run.
cudaError_t copy_heads(char* dev, char* host, bool to_dev, int B, int S, int h0, int hg, int D, size_t es,
                       const Strides3& hs, const ChunkLayout& L, cudaStream_t st) {
  const cudaMemcpyKind kind = cudaMemcpyDefault;
  const size_t row = (size_t)D * es;
  for (int b = 0; b < B; ++b) {
    char* hb = host + ((int64_t)b * hs.b + (int64_t)h0 * hs.h) * (int64_t)es;
    char* db = dev + (int64_t)b * L.st.b * (int64_t)es;
    cudaError_t e = cudaSuccess;
    if (L.token_major) {
      const size_t width = (size_t)hg * row, hp = (size_t)hs.s * es;
      e = to_dev ? cudaMemcpy2DAsync(db, width, hb, hp, width, S, kind, st)
                 : cudaMemcpy2DAsync(hb, hp, db, width, width, S, kind, st);
    } else if (hs.s == D && hs.h == (int64_t)S * D) {
      const size_t n = (size_t)hg * S * row;  // the chunk's heads are one contiguous run
      e = to_dev ? cudaMemcpyAsync(db, hb, n, kind, st) : cudaMemcpyAsync(hb, db, n, kind, st);
    } else {
      for (int h = 0; h < hg && e == cudaSuccess; ++h) {
        char* hh = hb + (int64_t)h * hs.h * (int64_t)es;
        char* dh = db + (int64_t)h * L.st.h * (int64_t)es;
        if (hs.s == D) {
          e = to_dev ? cudaMemcpyAsync(dh, hh, (size_t)S * row, kind, st)
                     : cudaMemcpyAsync(hh, dh, (size_t)S * row, kind, st);
        } else {
          const size_t hp = (size_t)hs.s * es;
          e = to_dev ? cudaMemcpy2DAsync(dh, row, hh, hp, row, S, kind, st)
                     : cudaMemcpy2DAsync(hh, hp, dh, row, row, S, kind, st);
        }
      }
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Staging bytes of one slot: the chunk's Q, K, V and output in the input dtype plus its LSE rows.
size_t slot_bytes(int B, int hg, int hkg, int Sq, int Skv, int D, size_t es) {
  return 2 * align256((size_t)B * Sq * hg * D * es) + 2 * align256((size_t)B * Skv * hkg * D * es) +
         align256((size_t)B * hg * Sq * 4);
}

// Chunk sizes in query heads for chunks of at most hg heads.  ramp 0: hg-head chunks (a shorter one
// first when hg does not divide H); 1: the last chunks shrink by halves (..., 4G, 2G, G), so that less
// attention and copy-out work is left once the last input has arrived; 2: the first chunks also grow by
// doubling (G, 2G, 4G, ...), so that the first kernels start sooner.
std::vector<int> chunk_sizes(int H, int G, int hg, int ramp) {
  const int u = hg / G;
  int rem = H / G;
  std::vector<int> front, back;
  if (ramp > 0)
    for (int x = 1; x < u; x *= 2) {
      const int take = ramp == 2 ? 2 * x : x;
      if (rem < take + u) break;  // keep at least one full chunk between the ramps
      back.push_back(x);
      if (ramp == 2) front.push_back(x);
      rem -= take;
    }
  if (rem % u) front.push_back(rem % u);
  std::sort(front.begin(), front.end());
  std::vector<int> out;
  for (int x : front) out.push_back(x * G);
  for (int i = 0; i < rem / u; ++i) out.push_back(hg);
  for (auto it = back.rbegin(); it != back.rend(); ++it) out.push_back(*it * G);
  return out;
}

// Time of the three-stage pipeline (copy in, compute, copy out, two staging slots) for the given chunk
// sizes, by event simulation.  The copies share one PCIe link: alone they run at the H2D / D2H rates,
// together at `both` split in that ratio.  A chunk's kernels take their CTAs' share of the GPU plus a
// per-chunk overhead, the last chunk's whole waves (the CTAs of the next chunk fill a partial wave).  The constants are measured on B200 (PCIe 5.0 x16; the Wan call's attention rate) and only
// rank the candidates: on the Wan call (B1 H40 N32760 D128) equal 1-, 2- and 4-head chunks take 23.4-23.5
// ms, 8-head chunks 23.9 ms, 20-head chunks 31.5 ms.
struct PipeModel {
  double q_bytes, kv_bytes, tiles_per_head, t_wave, nsm;
  int G;
};

PipeModel pipe_model(int B, int H, int Hkv, int Sq, int Skv, int D) {
  int dev = 0, nsm = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  if (nsm <= 0) nsm = 148;
  const double rate = 1.17e15;  // attention operations/s on a full GPU
  const double es = 2.0;
  const double rows = attention_rows_per_cta(D);
  PipeModel m;
  m.G = H / Hkv;
  m.nsm = nsm;
  m.tiles_per_head = (double)B * std::ceil(Sq / rows);
  const double t_head = 4.0 * B * Sq * (double)Skv * D / rate;  // one head's kernel time on a full GPU
  m.t_wave = t_head * nsm / m.tiles_per_head;                   // one full wave of CTAs
  m.q_bytes = (double)B * Sq * D * es;
  m.kv_bytes = 2.0 * B * Skv * D * es;
  return m;
}

double simulate_pipeline(const PipeModel& m, const std::vector<int>& sizes) {
  const double h2d = 51e9, d2h = 50e9, both = 88e9;  // bytes/s
  const double overhead = 70e-6;                      // per chunk: quantiser launches, ramp-up, copy set-up
  const int nch = (int)sizes.size();
  auto in_bytes = [&](int c) { return sizes[c] * m.q_bytes + (sizes[c] / m.G) * m.kv_bytes; };
  auto out_bytes = [&](int c) { return sizes[c] * m.q_bytes; };
  auto comp_time = [&](int c) {
    const double waves = sizes[c] * m.tiles_per_head / m.nsm;
    return overhead + (c == nch - 1 ? std::ceil(waves) : waves) * m.t_wave;
  };
  // chunk c's copy-in needs chunk c-2's kernels done (slot reuse); its kernels need its copy-in and chunk
  // c-2's copy-out done; its copy-out needs its kernels done
  std::vector<double> in_done(nch, -1), comp_done(nch, -1), out_done(nch, -1);
  int ci = 0, cc = 0, co = 0;
  double t = 0, in_rem = -1, out_rem = -1, comp_end = -1;
  for (int guard = 0; co < nch && guard < 8 * nch + 8; ++guard) {
    if (in_rem < 0 && ci < nch && (ci < 2 || (comp_done[ci - 2] >= 0 && comp_done[ci - 2] <= t)))
      in_rem = in_bytes(ci);
    if (comp_end < 0 && cc < nch && in_done[cc] >= 0 && in_done[cc] <= t &&
        (cc < 2 || (out_done[cc - 2] >= 0 && out_done[cc - 2] <= t)))
      comp_end = t + comp_time(cc);
    if (out_rem < 0 && co < nch && comp_done[co] >= 0 && comp_done[co] <= t) out_rem = out_bytes(co);
    const bool shared = in_rem >= 0 && out_rem >= 0;
    const double ri = shared ? both * h2d / (h2d + d2h) : h2d, ro = shared ? both * d2h / (h2d + d2h) : d2h;
    double dt = 1e30;
    if (in_rem >= 0) dt = std::min(dt, in_rem / ri);
    if (out_rem >= 0) dt = std::min(dt, out_rem / ro);
    if (comp_end >= 0) dt = std::min(dt, comp_end - t);
    if (dt >= 1e30) break;  // nothing can run (does not happen for a consistent schedule)
    t += dt;
    if (in_rem >= 0 && (in_rem -= ri * dt) <= 1.0) in_done[ci++] = t, in_rem = -1;
    if (out_rem >= 0 && (out_rem -= ro * dt) <= 1.0) out_done[co++] = t, out_rem = -1;
    if (comp_end >= 0 && comp_end <= t * (1 + 1e-12) + 1e-12) comp_done[cc++] = t, comp_end = -1;
  }
  return co == nch ? t : 1e30;
}

// The chunk plan: the largest chunk (query heads; 0 when hpc is not a multiple of the group size) and,
// when `sizes` is given, every chunk's size.  hpc > 0 fixes the largest chunk and the simulation picks
// the ramp; hpc <= 0 lets it pick both over every multiple of the group size.
int plan_chunks(int B, int H, int Hkv, int Sq, int Skv, int D, int hpc, std::vector<int>* sizes) {
  const int G = H / Hkv;
  if (hpc > 0 && hpc % G != 0) return 0;
  const PipeModel m = pipe_model(B, H, Hkv, Sq, Skv, D);
  const int lo = hpc > 0 ? std::min(hpc, H) / G : 1, hi = hpc > 0 ? lo : Hkv;
  int best_hg = lo * G, best_ramp = 0;
  double best_t = 1e30;
  for (int hkg = lo; hkg <= hi; ++hkg)
    for (int ramp = 0; ramp <= 2; ++ramp) {
      const double t = simulate_pipeline(m, chunk_sizes(H, G, hkg * G, ramp));
      if (t < best_t * 0.999) {
        best_t = t;
        best_hg = hkg * G;
        best_ramp = ramp;
      }
    }
  if (sizes != nullptr) *sizes = chunk_sizes(H, G, best_hg, best_ramp);
  return best_hg;
}

}  // namespace
}  // namespace sage

using namespace sage;

extern "C" {

int sage_host_heads_per_chunk(int B, int H, int Hkv, int Sq, int Skv, int D, int heads_per_chunk) {
  if (sage_qk_row_bytes(D) == 0 || B <= 0 || H <= 0 || Hkv <= 0 || H % Hkv != 0 || Sq <= 0 || Skv <= 0) return 0;
  return plan_chunks(B, H, Hkv, Sq, Skv, D, heads_per_chunk, nullptr);
}

int sage_host_chunk_plan(int B, int H, int Hkv, int Sq, int Skv, int D, int heads_per_chunk, int* sizes,
                         int max_chunks) {
  const int hg = sage_host_heads_per_chunk(B, H, Hkv, Sq, Skv, D, heads_per_chunk);
  if (hg == 0) return 0;
  std::vector<int> plan;
  plan_chunks(B, H, Hkv, Sq, Skv, D, hg, &plan);
  if (sizes != nullptr)
    for (int i = 0; i < (int)plan.size() && i < max_chunks; ++i) sizes[i] = plan[i];
  return (int)plan.size();
}

size_t sage_host_workspace_bytes(int B, int H, int Hkv, int Sq, int Skv, int D, int heads_per_chunk) {
  const int hg = sage_host_heads_per_chunk(B, H, Hkv, Sq, Skv, D, heads_per_chunk);
  if (hg == 0) return 0;
  const int hkg = hg / (H / Hkv);
  return 2 * slot_bytes(B, hg, hkg, Sq, Skv, D, 2) + 2 * align256(sage_workspace_bytes(B, hg, hkg, Sq, Skv, D));
}

int sage_attention_host(const void* q, const void* k, const void* v, int dtype, int B, int H, int Hkv, int Sq,
                        int Skv, int D, int64_t qsb, int64_t qss, int64_t qsh, int64_t ksb, int64_t kss, int64_t ksh,
                        int64_t vsb, int64_t vss, int64_t vsh, double sm_scale, int causal, void* out, int64_t osb,
                        int64_t oss, int64_t osh, float* lse, int heads_per_chunk, void* workspace,
                        size_t workspace_bytes, int* status, void* stream) {
  NvtxRange nvtx("sage_attention_host");
  if (dtype != SAGE_BF16 && dtype != SAGE_F16) {
    set_error("dtype %d (SAGE_BF16 or SAGE_F16 required)", dtype);
    return SAGE_ERR_UNSUPPORTED;
  }
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr) {
    set_error("q, k, v and out must be non-null");
    return SAGE_ERR_INVALID;
  }
  const int hg = sage_host_heads_per_chunk(B, H, Hkv, Sq, Skv, D, heads_per_chunk);
  std::vector<int> sizes;
  if (hg != 0) plan_chunks(B, H, Hkv, Sq, Skv, D, hg, &sizes);
  if (hg == 0) {
    set_error("unsupported sizes or heads_per_chunk %d (B=%d H=%d Hkv=%d Sq=%d Skv=%d D=%d)", heads_per_chunk, B, H,
              Hkv, Sq, Skv, D);
    return SAGE_ERR_UNSUPPORTED;
  }
  const size_t need = sage_host_workspace_bytes(B, H, Hkv, Sq, Skv, D, heads_per_chunk);
  if (workspace == nullptr || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u)) {
    set_error("workspace of %zu bytes (256-byte aligned) required, got %zu", need, workspace_bytes);
    return SAGE_ERR_INVALID;
  }
  const int G = H / Hkv, hkg = hg / G;
  const size_t es = 2;
  const Strides3 hq{qsb, qss, qsh}, hk{ksb, kss, ksh}, hv{vsb, vss, vsh}, ho{osb, oss, osh};
  // carve: slot 0, slot 1, then the quantised-tensor scratch of each slot (the chunks of the two slots
  // run on different streams)
  char* base = static_cast<char*>(workspace);
  struct Slot {
    char *q, *k, *v, *o;
    float* lse;
  } slot[2];
  size_t off = 0;
  for (int s = 0; s < 2; ++s) {
    slot[s].q = base + off;
    off += align256((size_t)B * Sq * hg * D * es);
    slot[s].k = base + off;
    off += align256((size_t)B * Skv * hkg * D * es);
    slot[s].v = base + off;
    off += align256((size_t)B * Skv * hkg * D * es);
    slot[s].o = base + off;
    off += align256((size_t)B * Sq * hg * D * es);
    slot[s].lse = reinterpret_cast<float*>(base + off);
    off += align256((size_t)B * hg * Sq * 4);
  }
  const size_t scratch_bytes = align256(sage_workspace_bytes(B, hg, hkg, Sq, Skv, D));
  char* scratch[2] = {base + off, base + off + scratch_bytes};

  std::lock_guard<std::mutex> lock(g_pipe_mu);
  int dev = 0;
  HostPipe* P = pipe_for_current_device(&dev);
  if (P == nullptr) {
    set_error("could not create the copy streams on the current device");
    return SAGE_ERR_LAUNCH;
  }
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  auto fail = [](cudaError_t e, const char* what) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return SAGE_ERR_LAUNCH;
  };
  cudaError_t e = cudaEventRecord(P->start, cs);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(P->in, P->start, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(P->out, P->start, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(P->comp, P->start, 0);
  if (e != cudaSuccess) return fail(e, "stream join");
  const int nch = (int)sizes.size();
  for (int c = 0, h0 = 0; c < nch; h0 += sizes[c], ++c) {
    const int s = c & 1, hc = sizes[c], kv0 = h0 / G, hkc = hc / G;
    Slot& S = slot[s];
    // copy in: the slot is free once chunk c-2's kernels have read it
    if (c >= 2) e = cudaStreamWaitEvent(P->in, P->comp_done[s], 0);
    if (e == cudaSuccess)
      e = copy_heads(S.q, (char*)q, true, B, Sq, h0, hc, D, es, hq, chunk_layout(hq, Sq, hc, D), P->in);
    if (e == cudaSuccess)
      e = copy_heads(S.k, (char*)k, true, B, Skv, kv0, hkc, D, es, hk, chunk_layout(hk, Skv, hkc, D), P->in);
    if (e == cudaSuccess)
      e = copy_heads(S.v, (char*)v, true, B, Skv, kv0, hkc, D, es, hv, chunk_layout(hv, Skv, hkc, D), P->in);
    if (e == cudaSuccess) e = cudaEventRecord(P->in_done[s], P->in);
    if (e != cudaSuccess) return fail(e, "copy in");
    // compute on the slot's stream, once the inputs are in and chunk c-2's output has left the slot (debug
    // builds keep every chunk on the caller's stream: their store checks read one table of the buffers the
    // current launches may write, which kernels of two chunks running at once would share)
#ifdef SAGE_DEBUG
    cudaStream_t ks = cs;
#else
    cudaStream_t ks = s == 0 ? cs : P->comp;
#endif
    e = cudaStreamWaitEvent(ks, P->in_done[s], 0);
    if (e == cudaSuccess && c >= 2) e = cudaStreamWaitEvent(ks, P->out_done[s], 0);
    if (e != cudaSuccess) return fail(e, "stream wait");
    const ChunkLayout cq = chunk_layout(hq, Sq, hc, D), ck = chunk_layout(hk, Skv, hkc, D),
                      cv = chunk_layout(hv, Skv, hkc, D), co = chunk_layout(ho, Sq, hc, D);
    int rc = sage_attention(S.q, S.k, S.v, dtype, B, hc, hkc, Sq, Skv, D, cq.st.b, cq.st.s, cq.st.h, ck.st.b, ck.st.s,
                            ck.st.h, cv.st.b, cv.st.s, cv.st.h, sm_scale, causal, S.o, co.st.b, co.st.s, co.st.h,
                            lse != nullptr ? S.lse : nullptr, scratch[s], scratch_bytes, status, ks);
    if (rc != SAGE_OK) return rc;
    e = cudaEventRecord(P->comp_done[s], ks);
    // copy out
    if (e == cudaSuccess) e = cudaStreamWaitEvent(P->out, P->comp_done[s], 0);
    if (e == cudaSuccess) e = copy_heads(S.o, (char*)out, false, B, Sq, h0, hc, D, es, ho, co, P->out);
    if (e == cudaSuccess && lse != nullptr)
      e = cudaMemcpy2DAsync(lse + (size_t)h0 * Sq, (size_t)H * Sq * 4, S.lse, (size_t)hc * Sq * 4,
                            (size_t)hc * Sq * 4, B, cudaMemcpyDefault, P->out);
    if (e == cudaSuccess) e = cudaEventRecord(P->out_done[s], P->out);
    if (e != cudaSuccess) return fail(e, "copy out");
  }
  // the caller's stream completes after the last output copy (the out stream runs its copies in order, each
  // after its chunk's kernels, so the second compute stream's work is done too)
  e = cudaStreamWaitEvent(cs, P->out_done[(nch - 1) & 1], 0);
  if (e != cudaSuccess) return fail(e, "stream join");
  return SAGE_OK;
}

// One device's share of a multi-device call: units u0 .. u1-1 of the flattened (batch, kv head) index,
// cut at batch boundaries into pieces of one batch and a range of kv heads.
struct Piece {
  int b, g0, g1;
};

static std::vector<Piece> device_pieces(int B, int Hkv, int n_dev, int d) {
  const int64_t units = (int64_t)B * Hkv;
  const int64_t u0 = units * d / n_dev, u1 = units * (d + 1) / n_dev;
  std::vector<Piece> out;
  for (int64_t u = u0; u < u1;) {
    const int b = (int)(u / Hkv), g0 = (int)(u % Hkv);
    const int g1 = (int)std::min<int64_t>(Hkv, g0 + (u1 - u));
    out.push_back({b, g0, g1});
    u += g1 - g0;
  }
  return out;
}

size_t sage_host_multi_workspace_bytes(int B, int H, int Hkv, int Sq, int Skv, int D, int heads_per_chunk,
                                       int n_devices) {
  if (n_devices <= 0 || B <= 0 || Hkv <= 0 || H % Hkv != 0) return 0;
  const int G = H / Hkv;
  size_t need = 0;
  for (int d = 0; d < n_devices; ++d)
    for (const Piece& pc : device_pieces(B, Hkv, n_devices, d)) {
      const int hkp = pc.g1 - pc.g0;
      const int hpc = heads_per_chunk > 0 ? std::min(heads_per_chunk, hkp * G) : 0;
      const size_t n = sage_host_workspace_bytes(1, hkp * G, hkp, Sq, Skv, D, hpc);
      if (n == 0) return 0;
      need = std::max(need, n);
    }
  return need;
}

int sage_attention_host_multi(const void* q, const void* k, const void* v, int dtype, int B, int H, int Hkv, int Sq,
                              int Skv, int D, int64_t qsb, int64_t qss, int64_t qsh, int64_t ksb, int64_t kss,
                              int64_t ksh, int64_t vsb, int64_t vss, int64_t vsh, double sm_scale, int causal,
                              void* out, int64_t osb, int64_t oss, int64_t osh, float* lse, int heads_per_chunk,
                              int n_devices, const int* devices, void* const* workspaces, size_t workspace_bytes,
                              int* const* statuses, void* const* streams) {
  NvtxRange nvtx("sage_attention_host_multi");
  if (n_devices <= 0 || devices == nullptr || workspaces == nullptr || streams == nullptr) {
    set_error("n_devices > 0 and device, workspace and stream arrays required");
    return SAGE_ERR_INVALID;
  }
  if (B <= 0 || H <= 0 || Hkv <= 0 || H % Hkv != 0) {
    set_error("sizes B=%d H=%d Hkv=%d (H a multiple of Hkv required)", B, H, Hkv);
    return SAGE_ERR_UNSUPPORTED;
  }
  const size_t need = sage_host_multi_workspace_bytes(B, H, Hkv, Sq, Skv, D, heads_per_chunk, n_devices);
  if (need == 0) {
    set_error("unsupported sizes or heads_per_chunk %d", heads_per_chunk);
    return SAGE_ERR_UNSUPPORTED;
  }
  if (workspace_bytes < need) {
    set_error("workspace of %zu bytes per device required, got %zu", need, workspace_bytes);
    return SAGE_ERR_INVALID;
  }
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) {
    set_error("cudaGetDevice failed");
    return SAGE_ERR_LAUNCH;
  }
  const int G = H / Hkv;
  const size_t es = 2;
  int rc = SAGE_OK;
  for (int d = 0; d < n_devices && rc == SAGE_OK; ++d) {
    const cudaError_t e = cudaSetDevice(devices[d]);
    if (e != cudaSuccess) {
      set_error("cudaSetDevice(%d): %s", devices[d], cudaGetErrorString(e));
      rc = SAGE_ERR_LAUNCH;
      break;
    }
    // the device's pieces run one after the other on its stream, reusing its workspace
    for (const Piece& pc : device_pieces(B, Hkv, n_devices, d)) {
      const int hkp = pc.g1 - pc.g0, hp = hkp * G, h0 = pc.g0 * G;
      const int hpc = heads_per_chunk > 0 ? std::min(heads_per_chunk, hp) : 0;
      const char* qp = static_cast<const char*>(q) + ((int64_t)pc.b * qsb + (int64_t)h0 * qsh) * (int64_t)es;
      const char* kp = static_cast<const char*>(k) + ((int64_t)pc.b * ksb + (int64_t)pc.g0 * ksh) * (int64_t)es;
      const char* vp = static_cast<const char*>(v) + ((int64_t)pc.b * vsb + (int64_t)pc.g0 * vsh) * (int64_t)es;
      char* op = static_cast<char*>(out) + ((int64_t)pc.b * osb + (int64_t)h0 * osh) * (int64_t)es;
      float* lp = lse != nullptr ? lse + ((int64_t)pc.b * H + h0) * Sq : nullptr;
      rc = sage_attention_host(qp, kp, vp, dtype, 1, hp, hkp, Sq, Skv, D, qsb, qss, qsh, ksb, kss, ksh, vsb, vss, vsh,
                               sm_scale, causal, op, osb, oss, osh, lp, hpc, workspaces[d], workspace_bytes,
                               statuses != nullptr ? statuses[d] : nullptr, streams[d]);
      if (rc != SAGE_OK) break;
    }
  }
  cudaSetDevice(prev);
  return rc;
}

}  // extern "C"
