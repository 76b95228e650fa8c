/*
 * b2gpu: C ABI of the B200 engine for AtlasIR (`atlasir-v1`) simulations.
 *
 * Drop-in boundary for the reference's execution core.  The reference runs its
 * engine as the `b2-runner MODEL.json OUTDIR` subprocess
 * (brian2-rust/src/model.rs:4596-4677, main.rs:2-7) over the Rust
 * `Runtime` (brian2-rust/src/executor.rs:3473-4824).  The entry points below
 * map one to one onto that runtime, and follow the in-tree C ABI precedent for
 * GPU offload (brian2-rust/python/brian2_rust/mpi_runtime/gpu_cuda.cpp:17-51,
 * loaded with dlopen/dlsym in mpi_runtime/gpu.rs:17-49):
 *   - an opaque handle; constructors return NULL on failure;
 *   - a caller-owned error buffer (char *error, size_t capacity), always
 *     NUL-terminated when capacity > 0;
 *   - int return codes: 0 success, non-zero failure;
 *   - plain C types only; one host thread per engine.
 * A failed engine is poisoned like the reference `Runtime` (executor.rs:
 * 3917-3925): every later call fails until it is destroyed.
 */
#ifndef B2GPU_H
#define B2GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2G_ABI_VERSION 1

typedef struct b2g_engine b2g_engine;

typedef struct b2g_options {
  uint32_t struct_size;   /* sizeof(b2g_options); lets the struct grow compatibly */
  int32_t device;         /* CUDA device ordinal, -1 for the current device */
  uint32_t chunk_ticks;   /* ticks per CUDA-graph replay, 0 for the default (128) */
  uint32_t use_graphs;    /* 1: replay captured graphs (default), 0: direct launches */
  uint64_t ring_capacity; /* spike-ring entries per event stream, 0 for automatic */
  /* Multi-GPU (one process per GPU).  Rank r of world_size owns the global
   * indices [floor(N*r/world_size), floor(N*(r+1)/world_size)) of every
   * population that a synapse targets, the reference's owner rule
   * ((i+1)*world_size-1)/N (brian2_rust/distributed.py:80-81,
   * mpi_codegen.py:40-44), and the incoming edges of its neurons; a
   * population that no synapse targets runs whole on every rank.  Callers
   * built against an older header pass a smaller struct_size and get
   * world_size 1. */
  int32_t rank;                 /* 0 .. world_size-1 */
  int32_t world_size;           /* number of GPUs/processes, 1 for a single GPU */
  uint32_t exchange_timeout_ms; /* bound on every wait for a peer's spikes, 0 for 10000 */
  uint32_t reserved0;
} b2g_options;

typedef struct b2g_stats {
  uint64_t ticks;              /* ticks simulated so far */
  uint64_t synaptic_events;    /* summary.json `synaptic_events` so far */
  uint64_t spikes;             /* events recorded on every stream so far */
  uint64_t kernel_launches;    /* launches of the engine's kernels so far */
  uint64_t launches_per_tick;  /* kernels per tick in the compiled plan */
  double simulation_seconds;   /* wall time inside b2g_step */
  double build_seconds;        /* b2g_create: device state, topology, compile */
  double compile_seconds;      /* NVRTC share of build_seconds */
  double device_seconds;       /* CUDA-event time of the tick kernels */
  uint64_t h2d_bytes;          /* host->device bytes moved by b2g_step */
  uint64_t d2h_bytes;          /* device->host bytes moved by b2g_step (spike drain) */
} b2g_stats;

typedef struct b2g_kernel_time {
  char name[64];
  uint64_t launches;
  double total_ms;
} b2g_kernel_time;

/* Fill `options` with defaults (struct_size set). */
void b2g_default_options(b2g_options* options);

/* Validate and load an AtlasIR document and build the device plan.
 * Replaces `Runtime::new` (executor.rs:3473) after `Model::validate`
 * (model.rs:3203).  Unsupported models fail here, before any result file
 * exists (brian2-rust/AtlasIR.md:66-70). */
b2g_engine* b2g_create(const char* json, size_t json_len, const b2g_options* options, char* error,
                       size_t error_capacity);

/* Advance at most `max_ticks` ticks; *finished is set to 1 when the run is
 * complete.  Replaces `Runtime::step` (executor.rs:3917). */
int b2g_step(b2g_engine* engine, uint64_t max_ticks, int* finished, char* error, size_t error_capacity);

/* Write results.bin (B2DMP001 v3), events.bin (B2EVT001, when the model has
 * event streams) and summary.json into the existing directory `outdir`.
 * Replaces `Runtime::write_results` plus the file writing of `execute`
 * (executor.rs:4749-4824). */
int b2g_write_results(b2g_engine* engine, const char* outdir, char* error, size_t error_capacity);

/* summary.json of a completed run as text, without writing files: *length
 * receives the text's size; when `buffer` is given, up to capacity - 1 bytes
 * and a NUL are copied.  dump_bytes / event_dump_bytes are the sizes
 * b2g_write_results would write; the recording time is 0.  Replaces the
 * summary of `execute` (executor.rs:4749-4824). */
int b2g_summary_json(b2g_engine* engine, char* buffer, size_t capacity, size_t* length, char* error,
                     size_t error_capacity);

int b2g_get_stats(const b2g_engine* engine, b2g_stats* stats, char* error, size_t error_capacity);

/* Advance `ticks` ticks launching every kernel directly, bracketed by CUDA
 * events on the engine's stream; fills up to `capacity` per-kernel records
 * (launch count, summed milliseconds) and sets *count.  No reference
 * counterpart: measurement support for the roofline report. */
int b2g_profile(b2g_engine* engine, uint64_t ticks, b2g_kernel_time* out, size_t capacity, size_t* count,
                char* error, size_t error_capacity);

/* Copy the raw storage bytes of a population state array (dtype width x
 * count); *needed receives the size.  Passing dst=NULL queries the size. */
int b2g_read_state(b2g_engine* engine, uint32_t population, const char* name, void* dst, size_t capacity,
                   size_t* needed, char* error, size_t error_capacity);

/* Ascending spike indices of `population` at absolute `tick`. */
int b2g_spikes(b2g_engine* engine, uint32_t population, uint64_t tick, uint32_t* dst, size_t capacity,
               size_t* count, char* error, size_t error_capacity);

/* The generated CUDA source of the compiled plan (diagnostics). */
int b2g_generated_source(const b2g_engine* engine, char* dst, size_t capacity, size_t* needed);

/* Build the plan of a model and compile its generated kernels for sm_100a
 * without a GPU; copies the generated source to dst (NULL queries *needed).
 * Same validation and capability errors as b2g_create. */
int b2g_codegen(const char* json, size_t json_len, const b2g_options* options, char* dst, size_t capacity,
                size_t* needed, char* error, size_t error_capacity);

/* ---- multi-GPU ------------------------------------------------------------
 * Replaces the reference's MPI exchange (brian2_rust/mpi_runtime/bridge.c:
 * 74-101: MPI_Allgather of counts + MPI_Allgatherv of global spike ids every
 * tick, rank 0 writing the results).  Here each engine's step kernel stores
 * every tile's spike list straight into every peer GPU's memory over NVLink
 * (and, where synaptic code reads a partitioned population's state, a
 * replicate kernel copies it the same way), so the host only takes part
 * once, to trade IPC handles:
 *   1. every rank: b2g_create with rank/world_size, then b2g_ipc_handle;
 *   2. the caller all-gathers the handles (any host transport: MPI, a
 *      torch.distributed store, ...) and every rank calls b2g_connect;
 *   3. b2g_step as usual (all ranks the same tick budgets);
 *   4. every rank: b2g_publish_results; the caller synchronises the ranks;
 *      rank 0: b2g_write_results (merged, identical to a one-GPU run).
 * b2g_read_state returns the rank's own block (all of a replicated
 * population, i.e. one that no synapse targets: every rank evaluates it
 * whole); b2g_spikes returns the global list of a population whose spikes
 * an on_pre pathway reads (every rank holds it), else the rank's own block's
 * (rank 0's results merge every rank's); b2g_get_stats counts this rank's
 * deliveries. */

/* Global index range [*lo, *hi) that `rank` of `world_size` owns in a
 * population of `count` neurons (pure function, no engine needed). */
void b2g_partition(uint64_t count, int32_t rank, int32_t world_size, uint64_t* lo, uint64_t* hi);

/* Opaque CUDA IPC handle of this engine's shared allocation (*length bytes,
 * at most 64). */
int b2g_ipc_handle(b2g_engine* engine, void* handle, size_t capacity, size_t* length, char* error,
                   size_t error_capacity);

/* Map the peers' allocations: `handles` is every rank's handle in rank order,
 * `count` = world_size handles of `handle_length` bytes each. */
int b2g_connect(b2g_engine* engine, const void* handles, size_t handle_length, size_t count, char* error,
                size_t error_capacity);

/* Stage this rank's final local results for rank 0 (after the last step). */
int b2g_publish_results(b2g_engine* engine, char* error, size_t error_capacity);

/* ---- device primitive ----------------------------------------------------
 * The reference's ascending `fired` list (emit_threshold, executor.rs:
 * 2949-3006) from a device bitmap with one bit per neuron (bit b of word w is
 * neuron 32*w + b; bits at or past nbits are ignored) -- the fired-word layout
 * of the engine's exchange between GPUs, for callers that evaluate thresholds
 * in their own kernels.  All pointers are device pointers; d_ids needs room
 * for the number of set bits; *d_count receives that number.  Asynchronous on
 * `stream` (a cudaStream_t; NULL is the legacy default stream).  d_scratch:
 * b2g_spikes_scratch_bytes(nbits) bytes of device memory, overwritten (it
 * needs no initialisation).  No engine involved. */
size_t b2g_spikes_scratch_bytes(uint64_t nbits);
int b2g_spikes_from_bitmap(const uint32_t* d_words, uint64_t nbits, uint32_t* d_ids, uint32_t* d_count,
                           void* d_scratch, size_t scratch_bytes, void* stream, char* error, size_t error_capacity);

/* No counterpart in the reference.  b2g_spikes_from_bitmap for callers that
 * cannot allocate device memory around the call (a tick loop that must not
 * stall on an allocator, a framework whose caching allocator holds the
 * device's memory budget, a process that has reserved all free memory): the
 * scratch is a fixed array inside the library, one per device, so
 *   - nbits must not exceed B2G_SPIKES_NOALLOC_MAX_BITS (else error 1);
 *   - calls whose launches overlap on one GPU race on that array;
 *   - the first call on a device does a one-time set-up (it looks the array
 *     up, which may load the library's device code), so make it before any
 *     stream capture; the set-up is repeated, in the same way, on the first
 *     call after the device's context was destroyed and re-created (for
 *     instance by cudaDeviceReset), because the array then has a new address;
 *   - the launches go to `stream`'s device, which the call makes current for
 *     its duration when another device is current.
 * Nothing needs to be zeroed beforehand. */
#define B2G_SPIKES_NOALLOC_MAX_BITS (1ull << 27)
int b2g_spikes_from_bitmap_noalloc(const uint32_t* d_words, uint64_t nbits, uint32_t* d_ids, uint32_t* d_count,
                                   void* stream, char* error, size_t error_capacity);

void b2g_destroy(b2g_engine* engine);

const char* b2g_version(void);

/* The complete `b2-runner` command line (argv[0] is ignored):
 *   MODEL.json OUTDIR | --validate MODEL.json
 * Same exit codes, stdout line and stderr prefix as model.rs:4596-4677. */
int b2g_run_cli(int argc, const char* const* argv);

#ifdef __cplusplus
}
#endif

#endif /* B2GPU_H */
