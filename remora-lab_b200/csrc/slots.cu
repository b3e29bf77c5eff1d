// slots.cu — expert-slot residency: a bounded table of device slots, each
// holding one projection (gate, up or down) of one expert, for deployments
// whose experts do not all stay resident (ExpertSlotTable,
// har/crates/har-vulkan/src/lib.rs:1233-1460; created by
// create_expert_slot_table, :925-970).
//
// The table is bookkeeping over one device allocation of count x slot_bytes:
// it records which key (layer, expert, projection, generation) occupies each
// slot and where the slot is in its life cycle,
//   Free -> Uploading (reserve) -> Ready (mark_ready, once the upload's event
//   has completed) -> InFlight (acquire_for_dispatch) -> Ready (release, once
//   the dispatch's event has completed) ... -> Free (evict, not while in flight),
// with a monotone epoch stamped on every transition (the caller's LRU order).
// The rules and their error cases follow the reference one for one; the
// reference's timeline-semaphore values become CUDA events (a cudaEvent_t
// passed as void*), complete when cudaEventQuery returns cudaSuccess.
// har_cuda_slot_upload is the B200 side of mark_upload_submitted: it copies a
// projection into its slot on the context's stream and records the event.
//
// A table created without a context has no storage: it is the state machine
// alone (the host side of a caller that moves the bytes itself), and its
// events must be NULL, meaning "already complete".  The kernels never see the
// table: a caller wraps a table's storage as Q4_K weights [count][N][K/256]
// (har_cuda_weights_wrap_q4k) and maps expert ids to slot ids, so one table
// per projection with matching slot indices serves an ordinary MoE layer.
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "har_internal.cuh"

struct SlotRecord {
  har_cuda_slot_snapshot snap;
  void *upload = nullptr;  // the event of the submitted upload (caller's or the table's)
  bool uploaded = false;   // an upload was submitted
  cudaEvent_t own = nullptr;  // the table's event for har_cuda_slot_upload
};

struct har_cuda_slot_table {
  har_cuda_ctx *ctx = nullptr;  // null: bookkeeping only
  void *storage = nullptr;
  uint64_t slot_bytes = 0;
  std::mutex mu;
  std::vector<SlotRecord> slots;
  uint64_t epoch = 1;  // the next epoch handed out (the reference starts at 1)
  std::string last_error;
};

namespace {

int32_t fail(har_cuda_slot_table *t, const char *what, const char *why,
             int32_t code = HAR_CUDA_ERR_ARG) {
  const std::string msg = std::string(what) + ": " + why;
  t->last_error = msg;
  if (t->ctx) har::set_error(t->ctx, code, msg);
  return code;
}

uint64_t next_epoch(har_cuda_slot_table *t) { return t->epoch++; }

int32_t on_device(har_cuda_ctx *ctx) {
  const cudaError_t e = cudaSetDevice(ctx->device);
  return e == cudaSuccess ? HAR_CUDA_OK
                          : har::set_error(ctx, HAR_CUDA_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
}

bool key_eq(const har_cuda_slot_key &a, const har_cuda_slot_key &b) {
  return a.layer == b.layer && a.expert_id == b.expert_id && a.projection == b.projection &&
         a.generation == b.generation;
}

// The event is complete.  A table without storage takes only NULL ("already
// complete"); one with storage takes a recorded cudaEvent_t.
int32_t event_done(har_cuda_slot_table *t, void *event, const char *what, const char *why) {
  if (!t->ctx) return event ? fail(t, what, "a table without storage takes NULL events") : HAR_CUDA_OK;
  if (!event) return fail(t, what, "event is null");
  const cudaError_t e = cudaEventQuery((cudaEvent_t)event);
  if (e == cudaSuccess) return HAR_CUDA_OK;
  if (e == cudaErrorNotReady) return fail(t, what, why);
  cudaGetLastError();
  return fail(t, what, cudaGetErrorString(e), HAR_CUDA_ERR_CUDA);
}

}  // namespace

extern "C" {

int32_t har_cuda_slot_table_create(har_cuda_ctx *ctx, uint32_t slot_count, uint64_t slot_bytes,
                                   har_cuda_slot_table **out) {
  if (!out) return HAR_CUDA_ERR_ARG;
  *out = nullptr;
  // create_expert_slot_table's check (lib.rs:930-936)
  if (slot_count == 0 || slot_bytes == 0 || slot_bytes > SIZE_MAX / slot_count)
    return ctx ? har::set_error(ctx, HAR_CUDA_ERR_ARG,
                                "create expert slot table: slot dimensions are zero or overflow host size")
               : HAR_CUDA_ERR_ARG;
  auto *t = new (std::nothrow) har_cuda_slot_table();
  if (!t) return HAR_CUDA_ERR_OOM;
  t->ctx = ctx;
  t->slot_bytes = slot_bytes;
  if (ctx) {
    int32_t st = on_device(ctx);
    if (st) {
      delete t;
      return st;
    }
    if (cudaMalloc(&t->storage, (size_t)slot_count * slot_bytes) != cudaSuccess) {
      cudaGetLastError();
      delete t;
      return har::set_error(ctx, HAR_CUDA_ERR_OOM, "create expert slot table: device allocation failed");
    }
  }
  t->slots.resize(slot_count);
  for (uint32_t i = 0; i < slot_count; ++i) {
    har_cuda_slot_snapshot &s = t->slots[i].snap;
    memset(&s, 0, sizeof(s));
    s.slot_id = i;
    s.state = HAR_CUDA_SLOT_FREE;
  }
  *out = t;
  return HAR_CUDA_OK;
}

int32_t har_cuda_slot_table_free(har_cuda_slot_table *t) {
  if (!t) return HAR_CUDA_OK;
  if (t->ctx) {
    on_device(t->ctx);
    // the storage may still be read or written by queued work
    cudaStreamSynchronize(t->ctx->stream);
    for (SlotRecord &r : t->slots)
      if (r.own) cudaEventDestroy(r.own);
    if (t->storage) cudaFree(t->storage);
  }
  delete t;
  return HAR_CUDA_OK;
}

int32_t har_cuda_slot_table_storage(har_cuda_slot_table *t, void **dev, uint64_t *bytes) {
  if (!t || !dev || !bytes) return HAR_CUDA_ERR_ARG;
  *dev = t->storage;
  *bytes = (uint64_t)t->slots.size() * t->slot_bytes;
  return HAR_CUDA_OK;
}

int32_t har_cuda_slot_table_last_error(const har_cuda_slot_table *t, char *buf, size_t len) {
  if (!t || !buf || len == 0) return HAR_CUDA_ERR_ARG;
  const size_t n = t->last_error.size() < len - 1 ? t->last_error.size() : len - 1;
  memcpy(buf, t->last_error.data(), n);
  buf[n] = '\0';
  return HAR_CUDA_OK;
}

// reserve (lib.rs:1282-1314)
int32_t har_cuda_slot_reserve(har_cuda_slot_table *t, const har_cuda_slot_key *key, uint32_t *slot_id) {
  if (!t || !key || !slot_id) return HAR_CUDA_ERR_ARG;
  std::lock_guard<std::mutex> g(t->mu);
  if (key->generation == 0) return fail(t, "reserve expert slot", "generation zero is reserved");
  if (key->projection > HAR_CUDA_PROJ_DOWN) return fail(t, "reserve expert slot", "unknown projection");
  for (const SlotRecord &r : t->slots)
    if (r.snap.state != HAR_CUDA_SLOT_FREE && key_eq(r.snap.key, *key))
      return fail(t, "reserve expert slot", "slot key is already resident or in flight");
  for (SlotRecord &r : t->slots) {
    if (r.snap.state != HAR_CUDA_SLOT_FREE) continue;
    const uint64_t e = next_epoch(t);
    r.snap.key = *key;
    r.snap.state = HAR_CUDA_SLOT_UPLOADING;
    r.snap.upload_epoch = e;
    r.snap.last_use_epoch = e;
    r.snap.ready = 0;
    r.upload = nullptr;
    r.uploaded = false;
    *slot_id = r.snap.slot_id;
    return HAR_CUDA_OK;
  }
  return fail(t, "reserve expert slot", "bounded slot table is full");
}

// mark_upload_submitted (lib.rs:1315-1333): the caller moved the bytes itself
int32_t har_cuda_slot_mark_upload_submitted(har_cuda_slot_table *t, uint32_t slot_id, void *event) {
  if (!t) return HAR_CUDA_ERR_ARG;
  std::lock_guard<std::mutex> g(t->mu);
  if (slot_id >= t->slots.size()) return fail(t, "mark expert upload", "slot ID is outside table");
  if (t->ctx ? !event : event != nullptr)
    return fail(t, "mark expert upload", t->ctx ? "event is null" : "a table without storage takes NULL events");
  SlotRecord &r = t->slots[slot_id];
  if (r.snap.state != HAR_CUDA_SLOT_UPLOADING) return fail(t, "mark expert upload", "slot is not awaiting upload");
  r.upload = event;
  r.uploaded = true;
  return HAR_CUDA_OK;
}

// The projection's bytes into the slot (an asynchronous copy on the context's
// stream), then mark_upload_submitted with the table's own event for the slot.
int32_t har_cuda_slot_upload(har_cuda_slot_table *t, uint32_t slot_id, const void *host_src, uint64_t bytes) {
  if (!t || !host_src) return HAR_CUDA_ERR_ARG;
  std::lock_guard<std::mutex> g(t->mu);
  if (!t->ctx) return fail(t, "upload expert slot", "the table has no storage");
  if (slot_id >= t->slots.size()) return fail(t, "upload expert slot", "slot ID is outside table");
  if (bytes == 0 || bytes > t->slot_bytes) return fail(t, "upload expert slot", "size exceeds the slot");
  SlotRecord &r = t->slots[slot_id];
  if (r.snap.state != HAR_CUDA_SLOT_UPLOADING) return fail(t, "upload expert slot", "slot is not awaiting upload");
  int32_t st = on_device(t->ctx);
  if (st) return st;
  if (!r.own && cudaEventCreateWithFlags(&r.own, cudaEventDisableTiming) != cudaSuccess) {
    cudaGetLastError();
    return fail(t, "upload expert slot", "event creation failed", HAR_CUDA_ERR_CUDA);
  }
  uint8_t *dst = static_cast<uint8_t *>(t->storage) + (size_t)slot_id * t->slot_bytes;
  cudaError_t e = cudaMemcpyAsync(dst, host_src, bytes, cudaMemcpyHostToDevice, t->ctx->stream);
  if (e == cudaSuccess) e = cudaEventRecord(r.own, t->ctx->stream);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(t, "upload expert slot", cudaGetErrorString(e), HAR_CUDA_ERR_CUDA);
  }
  r.upload = r.own;
  r.uploaded = true;
  return HAR_CUDA_OK;
}

// mark_ready (lib.rs:1334-1368).  event: the upload's event (NULL: the one
// recorded at submission); it must be the submitted one and complete.
int32_t har_cuda_slot_mark_ready(har_cuda_slot_table *t, uint32_t slot_id, void *event) {
  if (!t) return HAR_CUDA_ERR_ARG;
  std::lock_guard<std::mutex> g(t->mu);
  if (slot_id >= t->slots.size()) return fail(t, "mark expert ready", "slot ID is outside table");
  SlotRecord &r = t->slots[slot_id];
  if (r.snap.state != HAR_CUDA_SLOT_UPLOADING) return fail(t, "mark expert ready", "slot is not uploading");
  if (!r.uploaded) return fail(t, "mark expert ready", "slot has no submitted upload event");
  if (event && event != r.upload)
    return fail(t, "mark expert ready", "readiness event does not match upload event");
  int32_t st = event_done(t, r.upload, "mark expert ready", "upload event is not complete");
  if (st) return st;
  r.snap.state = HAR_CUDA_SLOT_READY;
  r.snap.ready = 1;
  r.upload = nullptr;
  r.uploaded = false;
  return HAR_CUDA_OK;
}

// acquire_for_dispatch (lib.rs:1369-1394)
int32_t har_cuda_slot_acquire(har_cuda_slot_table *t, const har_cuda_slot_key *key, har_cuda_slot_snapshot *out) {
  if (!t || !key || !out) return HAR_CUDA_ERR_ARG;
  std::lock_guard<std::mutex> g(t->mu);
  for (SlotRecord &r : t->slots) {
    if (!key_eq(r.snap.key, *key)) continue;
    if (r.snap.state != HAR_CUDA_SLOT_READY || !r.snap.ready)
      return fail(t, "acquire expert slot", "slot is not ready");
    r.snap.state = HAR_CUDA_SLOT_IN_FLIGHT;
    r.snap.last_use_epoch = next_epoch(t);
    *out = r.snap;
    return HAR_CUDA_OK;
  }
  return fail(t, "acquire expert slot", "projection-specific slot is not resident");
}

// release_from_dispatch (lib.rs:1395-1419): the dispatch's event has completed
int32_t har_cuda_slot_release(har_cuda_slot_table *t, uint32_t slot_id, void *event) {
  if (!t) return HAR_CUDA_ERR_ARG;
  std::lock_guard<std::mutex> g(t->mu);
  int32_t st = event_done(t, event, "release expert slot", "dispatch event is not complete");
  if (st) return st;
  if (slot_id >= t->slots.size()) return fail(t, "release expert slot", "slot ID is outside table");
  SlotRecord &r = t->slots[slot_id];
  if (r.snap.state != HAR_CUDA_SLOT_IN_FLIGHT) return fail(t, "release expert slot", "slot is not in flight");
  r.snap.state = HAR_CUDA_SLOT_READY;
  r.snap.ready = 1;
  r.snap.last_use_epoch = next_epoch(t);
  return HAR_CUDA_OK;
}

// evict (lib.rs:1420-1450): the completion event has completed; never in flight
int32_t har_cuda_slot_evict(har_cuda_slot_table *t, uint32_t slot_id, void *event) {
  if (!t) return HAR_CUDA_ERR_ARG;
  std::lock_guard<std::mutex> g(t->mu);
  int32_t st = event_done(t, event, "evict expert slot", "completion event is not complete");
  if (st) return st;
  if (slot_id >= t->slots.size()) return fail(t, "evict expert slot", "slot ID is outside table");
  SlotRecord &r = t->slots[slot_id];
  if (r.snap.state == HAR_CUDA_SLOT_IN_FLIGHT) return fail(t, "evict expert slot", "cannot evict an in-flight slot");
  r.snap.state = HAR_CUDA_SLOT_FREE;
  memset(&r.snap.key, 0, sizeof(r.snap.key));
  r.snap.ready = 0;
  r.snap.last_use_epoch = next_epoch(t);
  r.upload = nullptr;
  r.uploaded = false;
  return HAR_CUDA_OK;
}

// snapshot (lib.rs:1451-1456): every slot's record, in slot order
int32_t har_cuda_slot_table_snapshot(har_cuda_slot_table *t, har_cuda_slot_snapshot *out, uint32_t cap,
                                     uint32_t *n) {
  if (!t || !n || (cap && !out)) return HAR_CUDA_ERR_ARG;
  std::lock_guard<std::mutex> g(t->mu);
  *n = (uint32_t)t->slots.size();
  for (uint32_t i = 0; i < cap && i < *n; ++i) out[i] = t->slots[i].snap;
  return HAR_CUDA_OK;
}

}  // extern "C"
