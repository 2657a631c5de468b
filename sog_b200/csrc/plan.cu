// Plan utilities: buffers, errors, device guard, radix plans, version.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <string>

#include "plan.hpp"

namespace sogb {

static thread_local std::string g_last_error;

void set_error(const std::string &msg) { g_last_error = msg; }

int fail(int code, const std::string &msg) {
  g_last_error = msg;
  return code;
}

int DevBuf::reserve(size_t need) {
  if (need <= bytes && p) return SOG_OK;
  release();
  if (need == 0) need = 16;
  const size_t rounded = (need + 255) & ~size_t(255);
  if (cudaMalloc(&p, rounded) != cudaSuccess) {
    cudaGetLastError();
    p = nullptr;
    bytes = 0;
    g_last_error = "cudaMalloc of " + std::to_string(rounded) + " bytes failed";
    return SOG_ERR_NOMEM;
  }
  bytes = rounded;
  return SOG_OK;
}

void DevBuf::release() {
  if (p) cudaFree(p);
  p = nullptr;
  bytes = 0;
}

int PinnedBuf::reserve(size_t need) {
  if (!done) {
    if (cudaEventCreateWithFlags(&done, cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      return fail(SOG_ERR_CUDA, "cudaEventCreate failed");
    }
  }
  if (need <= bytes && p) return SOG_OK;
  if (int rc = wait()) return rc;
  if (p) cudaFreeHost(p);
  p = nullptr;
  bytes = 0;
  const size_t rounded = (need + 4095) & ~size_t(4095);
  if (cudaMallocHost(&p, rounded) != cudaSuccess) {
    cudaGetLastError();
    p = nullptr;
    return fail(SOG_ERR_NOMEM, "cudaMallocHost failed");
  }
  bytes = rounded;
  return SOG_OK;
}

int PinnedBuf::wait() {
  if (pending && done) {
    if (cudaEventSynchronize(done) != cudaSuccess) {
      cudaGetLastError();
      return fail(SOG_ERR_CUDA, "cudaEventSynchronize failed");
    }
  }
  pending = false;
  return SOG_OK;
}

void PinnedBuf::release() {
  wait();
  if (p) cudaFreeHost(p);
  if (done) cudaEventDestroy(done);
  p = nullptr;
  done = nullptr;
  bytes = 0;
}

DeviceGuard::DeviceGuard(int dev) {
  if (cudaGetDevice(&prev) != cudaSuccess) { cudaGetLastError(); prev = -1; }
  if (prev != dev) cudaSetDevice(dev);
}

DeviceGuard::~DeviceGuard() {
  int cur = -1;
  if (cudaGetDevice(&cur) == cudaSuccess && prev >= 0 && cur != prev) cudaSetDevice(prev);
}

// Radix sequence: eights first (fewest smem stages), then 4, 2, 3, 5.
void build_radix_plan(int n, RadixPlan *rp) {
  rp->n = n;
  rp->nst = 0;
  int m = n;
  while (m % 8 == 0 && m > 8) { rp->r[rp->nst++] = 8; m /= 8; }
  if (m == 8) { rp->r[rp->nst++] = 8; m = 1; }
  while (m % 4 == 0) { rp->r[rp->nst++] = 4; m /= 4; }
  while (m % 2 == 0) { rp->r[rp->nst++] = 2; m /= 2; }
  while (m % 3 == 0) { rp->r[rp->nst++] = 3; m /= 3; }
  while (m % 5 == 0) { rp->r[rp->nst++] = 5; m /= 5; }
  int ns = 1;
  for (int s = 0; s < rp->nst; ++s) {
    rp->nR[s] = n / rp->r[s];
    rp->Ns[s] = ns;
    rp->m_nR[s] = fdiv_mul((uint32_t)rp->nR[s]);
    rp->m_Ns[s] = fdiv_mul((uint32_t)ns);
    ns *= rp->r[s];
  }
}

static std::atomic<unsigned long long> g_launches{0};

void count_launch(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }

// Marks accumulate over calls until read (sog_plan_timings), so a whole timed
// region can be read once at its end; "begin" separates calls.
void Tracer::begin(cudaStream_t st) {
  if (!on) return;
  mark(st, "begin");
}

void Tracer::mark(cudaStream_t st, const char *name) {
  if (!on || used >= 65536) return;
  if (used >= (int)ev.size()) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) { cudaGetLastError(); return; }
    ev.push_back(e);
    names.push_back(nullptr);
  }
  names[used] = name;
  // inside a stream capture a plain record only orders captured streams;
  // the external flag makes it an event-record node of the graph
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess) cudaGetLastError();
  if (cs == cudaStreamCaptureStatusActive)
    cudaEventRecordWithFlags(ev[used], st, cudaEventRecordExternal);
  else
    cudaEventRecord(ev[used], st);
  ++used;
}

void Tracer::release() {
  for (cudaEvent_t e : ev) cudaEventDestroy(e);
  ev.clear();
  names.clear();
  used = 0;
}

}  // namespace sogb

extern "C" unsigned long long sog_launch_count(void) { return sogb::g_launches.load(); }

// Durations between consecutive marks of each call since the last read;
// clears the marks.
static int timings_of(sogb::Tracer &tr, const char **names, float *ms, int cap, int *count) {
  *count = 0;
  if (tr.used < 2) { tr.used = 0; return SOG_OK; }
  if (cudaEventSynchronize(tr.ev[tr.used - 1]) != cudaSuccess) {
    cudaGetLastError();
    return sogb::fail(SOG_ERR_CUDA, "cudaEventSynchronize failed");
  }
  int n = 0;
  for (int i = 1; i < tr.used && n < cap; ++i) {
    if (std::strcmp(tr.names[i], "begin") == 0) continue;
    float t = 0.f;
    cudaEventElapsedTime(&t, tr.ev[i - 1], tr.ev[i]);
    if (names) names[n] = tr.names[i];
    if (ms) ms[n] = t;
    ++n;
  }
  tr.used = 0;
  *count = n;
  return SOG_OK;
}

// A pool of events is created when timing is switched on, so that none is
// created inside the calls being timed.
static void tracer_reserve(sogb::Tracer &tr, int n) {
  while ((int)tr.ev.size() < n) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) { cudaGetLastError(); return; }
    tr.ev.push_back(e);
    tr.names.push_back(nullptr);
  }
}

extern "C" int sog_plan_set_timing(sog_plan *p, int on) {
  if (!p) return sogb::fail(SOG_ERR_INVALID, "null plan");
  p->tr.on = on != 0;
  p->tr.used = 0;
  if (p->tr.on) {
    sogb::DeviceGuard dg(p->d.device);
    tracer_reserve(p->tr, on > 2048 ? on : 2048);
  }
  return SOG_OK;
}

extern "C" int sog_plan_timings(sog_plan *p, const char **names, float *ms, int cap, int *count) {
  if (!p || !count) return sogb::fail(SOG_ERR_INVALID, "null argument");
  sogb::DeviceGuard dg(p->d.device);
  return timings_of(p->tr, names, ms, cap, count);
}

extern "C" int sog_direct_set_timing(sog_direct *d, int on) {
  if (!d) return sogb::fail(SOG_ERR_INVALID, "null context");
  d->tr.on = on != 0;
  d->tr.used = 0;
  if (d->tr.on) {
    sogb::DeviceGuard dg(d->device);
    tracer_reserve(d->tr, on > 2048 ? on : 2048);
  }
  return SOG_OK;
}

extern "C" int sog_direct_timings(sog_direct *d, const char **names, float *ms, int cap, int *count) {
  if (!d || !count) return sogb::fail(SOG_ERR_INVALID, "null argument");
  sogb::DeviceGuard dg(d->device);
  return timings_of(d->tr, names, ms, cap, count);
}

void sogb_set_cuda_error(cudaError_t e) {
  sogb::set_error(std::string("CUDA error: ") + cudaGetErrorString(e));
}

extern "C" const char *sog_strerror(int code) {
  switch (code) {
    case SOG_OK: return "ok";
    case SOG_ERR_INVALID: return "invalid argument";
    case SOG_ERR_CUDA: return "CUDA runtime error";
    case SOG_ERR_NOMEM: return "out of memory";
    case SOG_ERR_UNSUPPORTED: return "unsupported";
    case SOG_ERR_DEVICE: return "device status raised";
    case SOG_ERR_COMM: return "exchange callback failed";
    default: return "unknown error";
  }
}

extern "C" const char *sog_last_error(void) { return sogb::g_last_error.c_str(); }

extern "C" const char *sog_version(void) { return "sog_b200 0.1 (sm_100a)"; }
