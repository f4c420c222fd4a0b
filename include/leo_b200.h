/*
 * leo_b200: B200-native (sm_100a) per-byte training step over Leo's logical
 * story workers, behind a C ABI with plain pointers and sizes.
 *
 * Every entry point returns 0 on success and -1 on failure, with the message
 * available from leo_b200_last_error() (thread-local), mirroring LeoResult /
 * LeoError (crates/leo-core/src/lib.rs:43-55).  Explicit GPU selection never
 * falls back to a CPU path (crates/leo-core/src/backend.rs:803-822): without a
 * Blackwell device leo_b200_open fails.
 *
 * Types: include/leo_b200_types.h; kernel configuration layout: the generated
 * include/leo_cuda_abi.h (from cuda_abi.def, crates/leo-core/build.rs:97-121).
 */
#ifndef LEO_B200_H
#define LEO_B200_H

#include "leo_b200_types.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct LeoB200Device LeoB200Device;

/* Last error message of the calling thread (LeoError::message). */
const char* leo_b200_last_error(void);

/* LEO_CUDA_ABI_VERSION of the generated header; must equal the host's
   CUDA_ABI_VERSION (crates/leo-core/src/semantics.rs:12). */
uint32_t leo_b200_abi_version(void);

/* Config::validate (crates/leo-core/src/config.rs:250-519) plus this
   backend's device limits. */
int leo_b200_config_validate(const LeoB200Config* config);

/* Model::initialize (crates/leo-core/src/model.rs:79-158) into caller-owned
   arrays sized from the config; `topology` is a LeoB200Topology. */
int leo_b200_model_initialize(const LeoB200Config* config, int topology, LeoB200HostModel* model);

/* Model::validate (crates/leo-core/src/model.rs:223-396). */
int leo_b200_model_validate(const LeoB200HostModel* model);

/* training_state_hash (crates/leo-cli/src/main.rs:1187-1202) of a host model. */
int leo_b200_training_state_hash(const LeoB200HostModel* model, uint8_t out[32]);

/* Opens a backend on CUDA device `device` with `model` as the canonical
   model and room for `max_lanes` story lanes.  Replaces GpuRuntime::new /
   CudaRuntime creation (crates/leo-core/src/backend.rs:547-580,
   crates/leo-core/src/cuda.rs:1138-1207). */
int leo_b200_open(int device, const LeoB200HostModel* model, uint32_t max_lanes, LeoB200Device** out);
void leo_b200_close(LeoB200Device* device);

/* Replaces the canonical model and every resident lane
   (RuntimeBackend::model_mut + synchronize, backend.rs:355-357). */
int leo_b200_upload_canonical(LeoB200Device* device, const LeoB200HostModel* model);

/* RuntimeBackend::synchronize_model + model (backend.rs:355-356): copies the
   canonical model into caller-owned arrays (checkpoint layout). */
int leo_b200_download_model(LeoB200Device* device, LeoB200HostModel* model);

/* The canonical runtime's tick (Runtime::current_tick, runtime.rs:117); it
   advances with single-story and replay steps. */
uint64_t leo_b200_canonical_tick(LeoB200Device* device);
int leo_b200_set_canonical_tick(LeoB200Device* device, uint64_t tick);

/* One logical story batch: RuntimeBackend::training_story_batch
   (backend.rs:457-463) followed by the batch-end mean merge
   (parallel.rs:694-798) and serial canonical replay
   (crates/leo-cli/src/training.rs:1539-1727).  Stories are
   bytes[offsets[i] .. offsets[i+1]].  `summaries` (optional) receives one
   DeviceStorySummary per story, `losses` (optional) the initial-pass loss of
   every target of every story in story order (sum of len+1 floats). */
int leo_b200_train_story_batch(LeoB200Device* device, const uint8_t* bytes, const uint64_t* offsets,
                               uint32_t stories, int permission, LeoB200BatchReport* report,
                               LeoB200StorySummary* summaries, float* losses);

/* The same batch in three calls, so a caller can inspect lanes between steps:
   begin (lane reset + schedules), steps (advance `count` ticks), finish
   (remaining ticks, merge, replay, lane sync). */
int leo_b200_batch_begin(LeoB200Device* device, const uint8_t* bytes, const uint64_t* offsets, uint32_t stories,
                         int permission);
int leo_b200_batch_steps(LeoB200Device* device, uint32_t count, uint32_t* steps_done);
int leo_b200_batch_finish(LeoB200Device* device, LeoB200BatchReport* report, LeoB200StorySummary* summaries,
                          float* losses);

/* One logical batch sharded over several devices (exact data parallelism,
   MultiGpuBatchTrainer::train_story_batch, crates/leo-cli/src/training.rs:
   1212-1420, with its default serial canonical replay).  Every rank passes the
   whole batch and runs stories [first, first + count) on its lanes; the caller
   exchanges the merge between the rank-local steps (leo_b200/parallel.py does
   it over torch.distributed / NCCL):
     shard_begin, shard_local (this rank's story reports, losses and keyed
     context deltas), then for each fixed tensor t < LEO_B200_FIXED_TENSORS:
       shard_marks     element marks of this rank's lanes (device buffer of
                       shard_tensor_elements bytes), MAX-all-reduced by the caller
       shard_plan      sorted merge list from the reduced marks -> count
       shard_accumulate  partial[count] (FP64, device): rank 0 starts from 0.0,
                       rank r > 0 adds to the sums received from rank r - 1
       shard_finalize  last rank: merged values (f32, device) from the sums
       shard_commit    every rank: the broadcast values into the canonical
                       tensor and every resident lane
     shard_finish with every story's report, losses and context deltas in
     story order: keyed context merge, statistics, revision, the serial replay
     of every story (identical on every rank) and the report.
   One GPU running the whole batch and N ranks running its shards end with the
   same training_state_hash.  A batch of one story is not sharded (use
   leo_b200_train_story_batch on every rank). */
int leo_b200_shard_begin(LeoB200Device* device, const uint8_t* bytes, const uint64_t* offsets, uint32_t stories,
                         uint32_t first, uint32_t count, int permission);
int leo_b200_shard_local(LeoB200Device* device, LeoB200ShardStory* stories, float* losses, size_t* context_bytes);
int leo_b200_shard_context(LeoB200Device* device, uint8_t* out, size_t capacity);
int leo_b200_shard_tensor_elements(LeoB200Device* device, uint32_t tensor, size_t* elements);
int leo_b200_shard_marks(LeoB200Device* device, uint32_t tensor, uint8_t* marks);
int leo_b200_shard_plan(LeoB200Device* device, uint32_t tensor, const uint8_t* marks, uint32_t* count);
int leo_b200_shard_accumulate(LeoB200Device* device, uint32_t tensor, double* partial, int first);
int leo_b200_shard_finalize(LeoB200Device* device, uint32_t tensor, const double* partial, float* values);
int leo_b200_shard_commit(LeoB200Device* device, uint32_t tensor, const float* values);
int leo_b200_shard_finish(LeoB200Device* device, const LeoB200ShardStory* stories, const float* losses,
                          const uint8_t* context, const uint64_t* context_offsets, uint64_t fixed_updates,
                          LeoB200BatchReport* report, LeoB200StorySummary* summaries, float* losses_out);

/* ---- RuntimeBackend, trait-shaped (crates/leo-core/src/backend.rs:351-475) ----
   The entry points below let a caller drive the reference trainer's own loop
   (crates/leo-cli/src/training.rs:1584-1660, 1833-1945) step by step: a
   device story batch without replay, then the serial replay through the
   canonical runtime's document calls with parameter tracking, then the
   packed sparse sync.  Driven that way they reproduce the fused
   leo_b200_train_story_batch bit for bit. */

/* RuntimeBackend::training_story_batch (backend.rs:457-463, GpuRuntime
   backend.rs:739-764): every story on its own lane, the device-local mean
   merge into the canonical model and every lane; no replay.  Returns
   LEO_B200_UNSUPPORTED for fewer than two stories (backend.rs:587-589).
   `summaries` and `losses` as for leo_b200_train_story_batch; `range_counts`
   (optional, one per story) and `ranges` (optional, 2 x total ranges: start,
   end) receive each story's replay ranges (DeviceStoryBatchReport::
   replay_ranges, select_replay_ranges training.rs:1782-1830). */
int leo_b200_training_story_batch(LeoB200Device* device, const uint8_t* bytes, const uint64_t* offsets,
                                  uint32_t stories, int permission, LeoB200BatchReport* report,
                                  LeoB200StorySummary* summaries, float* losses, uint64_t* ranges,
                                  uint32_t* range_counts);

/* RuntimeBackend::training_story_batch_deltas (backend.rs:468-474,
   backend.rs:766-795): every story on its own lane (one story too); each
   story's private delta against the canonical model is kept for
   leo_b200_story_deltas (SparseModelDelta, from_tracked_values
   parallel.rs:461-674: changed indices with a nonzero difference, sorted; the
   output weights indexed output * neuron_count + neuron) and the lanes return
   to the canonical model, which this call does not change.  `sizes` receives
   the entry counts the caller allocates for. */
int leo_b200_training_story_batch_deltas(LeoB200Device* device, const uint8_t* bytes, const uint64_t* offsets,
                                         uint32_t stories, int permission, LeoB200BatchReport* report,
                                         LeoB200StorySummary* summaries, float* losses, uint64_t* ranges,
                                         uint32_t* range_counts, LeoB200StoryDeltaSizes* sizes);
/* The deltas of the last leo_b200_training_story_batch_deltas, into caller
   buffers sized from its LeoB200StoryDeltaSizes (NULL members are skipped). */
int leo_b200_story_deltas(LeoB200Device* device, const LeoB200StoryDeltas* out);

/* The canonical runtime's document (Runtime::begin_document /
   reset_transient_state, runtime.rs:353-435; backend.rs:391-402): the
   transient state is reset at the canonical tick; parameters, tracking and
   statistics are kept.  A story batch ends an open document. */
int leo_b200_begin_document(LeoB200Device* device);
int leo_b200_reset_transient_state(LeoB200Device* device);

/* RuntimeBackend::training_step_batch (backend.rs:413-421): `count` serial
   steps of the open document on the canonical model, step i reading input
   symbol symbols[i] (0..257) with target targets[i] (0..255 or 257;
   -1: none) at `permission`, in one device launch.  `losses` (optional)
   receives each step's loss (0 without a target), `active_neurons`
   (optional) its active-neuron count.  Advances the canonical tick,
   statistics and revision as Runtime::step does. */
int leo_b200_training_step_batch(LeoB200Device* device, const uint32_t* symbols, const int32_t* targets,
                                 uint32_t count, int permission, float* losses, uint32_t* active_neurons);

/* RuntimeBackend::advance_frozen_batch (backend.rs:428-431): the same steps
   at Permission::Frozen, metrics discarded. */
int leo_b200_advance_frozen_batch(LeoB200Device* device, const uint32_t* symbols, const int32_t* targets,
                                  uint32_t count);

/* Parameter tracking of the canonical runtime (RuntimeBackend::
   enable_parameter_tracking / parameter_changes, backend.rs:358-359; the
   CUDA backend's window semantics, cuda.rs:2827-2842): enabling starts an
   empty window (rows changed before it are first written into every lane);
   the window collects every index the canonical runtime's steps change
   (leo_b200_training_step_batch, leo_b200_advance_frozen_batch) and closes
   at the next story batch or packed sync, which write those rows into every
   lane.  leo_b200_parameter_changes stores the sizes and, when
   `changes` is not NULL, the sorted indices into its caller buffers. */
int leo_b200_enable_parameter_tracking(LeoB200Device* device);
int leo_b200_parameter_changes(LeoB200Device* device, LeoB200ParameterChangeSizes* sizes,
                               const LeoB200ParameterChanges* changes);

/* RuntimeBackend::synchronize_packed_model (backend.rs:374-376;
   PackedSparseModelUpdate::apply_to_model parallel.rs:196-300, the CUDA
   backend's device scatter cuda.rs:2869-3080): the packet's values written
   over the canonical model and every resident lane; generation, revision and
   statistics replaced.  Indices are validated before anything is written. */
int leo_b200_synchronize_packed_model(LeoB200Device* device, const LeoB200PackedUpdate* update);

/* RuntimeBackend::commit_packed_host_model (backend.rs:385-387; cuda.rs:
   2858-2867): the same writes, keeping the parameter-tracking window open
   (its tracked rows are written into the lanes at the next story batch). */
int leo_b200_commit_packed_host_model(LeoB200Device* device, const LeoB200PackedUpdate* update);

/* training_state_hash of the canonical device model. */
int leo_b200_state_digest(LeoB200Device* device, uint8_t out[32]);

/* Inspection for parity tests: a lane's learned parameters (lane ==
   UINT32_MAX: the canonical model) and its transient arrays by the reference
   runtime's field names (runtime.rs:112-186). */
int leo_b200_lane_model(LeoB200Device* device, uint32_t lane, LeoB200HostModel* model);
int leo_b200_lane_array(LeoB200Device* device, uint32_t lane, const char* name, void* out, size_t capacity,
                        size_t* written);

/* Performance counters (LeoB200PerfStats): kernel launches, work units per
   phase, per-phase clock counters and CUDA-event time of the wavefront
   launches, as the reference's phase profiler reports
   (crates/leo-core/src/cuda.rs:6998, cuda_kernels.cu:5764-5789). */
int leo_b200_perf_stats(LeoB200Device* device, LeoB200PerfStats* out);
int leo_b200_reset_perf_stats(LeoB200Device* device);

/* Execution geometry only (results do not depend on it): CTAs per thread-block
   cluster for story lanes and for the canonical replay lane; 0 picks the
   default (story: re-divided by lane load, see leo_b200_set_story_chunk;
   replay: a 16-CTA cluster, or the whole GPU -- one CTA per SM with grid-wide
   phase barriers -- when the replay lane's last reported work per step is
   large).  LEO_B200_WHOLE_GPU forces the whole-GPU replay launch.  The reference's
   execution tuner chooses the analogous geometry (crates/leo-core/src/cuda_plan.rs:189-453). */
int leo_b200_set_cluster_sizes(LeoB200Device* device, uint32_t story_cluster, uint32_t replay_cluster);

/* Execution geometry only: with the default story cluster size (0), the story
   pass runs in launches of `steps` steps (default 32; four times that while
   the lanes' loads are within 3x of the median), and before each launch
   the SMs are re-divided among the lanes that still have steps, in proportion
   to the work per step each lane reported (the reference's execution tuner
   plays this role statically, crates/leo-core/src/cuda_plan.rs:189-453). */
int leo_b200_set_story_chunk(LeoB200Device* device, uint32_t steps);

/* Where a one-GPU batch's keyed context merge runs: 1 (the default when a
   context order's slots fit 200 KB of shared memory at 17 bytes a slot) on the
   device, 0 on the host mirror.  Results are identical; the reference merges
   on the host (crates/leo-core/src/parallel.rs:1024-1113, cuda.rs:9230-9260). */
int leo_b200_set_device_context_merge(LeoB200Device* device, int enable);

/* Execution geometry only (results never depend on it).  Every target's
   events of a step are keys in its own segment, sorted and summed in event
   order by settle: by one thread when a step brings it at most
   `thread_events` events (1..16; 0: 16), by a warp up to 256, by a whole CTA
   above.  Targets whose recurrent in-degree is at least `min_in_degree` are
   listed (0 restores the default, max(1, 16 x neuron_count /
   (4 x max_active_global))): they are dealt over the CTAs in descending
   segment capacity, and among the first 512 those with more than
   `cta_events` events in the step (1..2048; 0: 256) are sorted one per CTA
   while the other CTAs settle the touched list.  Only before the first story
   batch.  leo_b200_hub_count reports the number of listed targets and the
   event-segment entries per lane. */
int leo_b200_set_hub_threshold(LeoB200Device* device, uint32_t min_in_degree, uint32_t cta_events,
                               uint32_t thread_events);
int leo_b200_hub_count(LeoB200Device* device, uint32_t* hubs, uint64_t* events_per_lane);

/* Diagnostic: caps every target's per-step event segment at `limit` entries
   (0: the exact bound, min(in-degree, 4 x max_active_global x multiplicity)
   plus the input fan-in, which no step can exceed).  A step whose events
   overrun a capped segment drops the extra events without writing past it
   and the batch fails with an error, as a device capacity overrun would.
   Only before the first story batch. */
int leo_b200_set_segment_capacity_limit(LeoB200Device* device, uint32_t limit);

/* Device memory held by the backend, in bytes. */
size_t leo_b200_device_bytes(LeoB200Device* device);

/* Batch-end sparse mean apply of one FP32 tensor plus the sync of its
   replicas, on device memory the caller owns: apply_sparse_scaled
   (crates/leo-core/src/parallel.rs:975-1022) with divisor = `stories`, then the
   clamp projection of parallel.rs:1226-1233 ([lo, hi]; pass -inf/+inf for
   none), then the merged values written into each of `replica_count` replica
   copies (the packed-update scatter, crates/leo-core/src/cuda.rs:2869-3080).
   Story s owns entries story_offsets[s] .. story_offsets[s + 1] of `indices`
   (sorted, strictly increasing, < length) and `deltas` (finite); the offsets
   and the replica pointer table are HOST arrays, everything else is device
   memory on `device`.  Invalid input (an index out of range or out of order,
   a non-finite delta) is rejected before anything is written.  A merged value
   that becomes non-finite is reported only after the merge pass: by then the
   target and the replicas may be partly updated (clamped values written for
   some tiles), as the reference's apply also fails after partial writes.
   At most 256 stories and 64 replicas per call.  `stream` is a cudaStream_t
   (NULL: the legacy default stream); the call waits for it and stores the
   number of merged indices in *updates.  Scratch (a tile table of
   stories x (length / 4096 + 1) words) is allocated on first use per device
   and kept; calls on one device are serialised. */
int leo_b200_sparse_mean_apply(int device, float* target, uint32_t length, const uint32_t* indices,
                               const float* deltas, const uint64_t* story_offsets, uint32_t stories, float lo,
                               float hi, float* const* replicas, uint32_t replica_count, void* stream,
                               uint32_t* updates);

/* The same apply with NO device allocation: no counterpart in the reference
   (which allocates its scratch with cuMemAlloc).  For callers that must not
   allocate device memory inside the call: cudaFree synchronises the whole
   device (stalling every other stream, NCCL's included), a process whose HBM
   is already reserved by a caching allocator can fail a fresh cudaMalloc for
   a small scratch, and latency-bounded loops must not enter the allocator.
   Scratch is a fixed 1 MiB device array compiled into the library: the call
   accepts stories * (ceil(length / 4096) + 1) <= 262080 (for example 63
   stories at length 2^24, or 256 stories up to length 4,186,112 = 1022
   tiles) and rejects larger inputs with an error before any device work; the
   other limits, the results and the error behaviour (including the partial
   writes before a non-finite merged value is reported) are those of
   leo_b200_sparse_mean_apply.  The first call on a device resolves the
   array's address (cudaGetSymbolAddress); make that first call before any
   stream capture begins.  Every call zeroes the counters at
   the head of the array on `stream` before its kernels run.  All calls on one
   device share the array: calls that overlap in time race, so the caller
   serialises them. */
int leo_b200_sparse_mean_apply_static(int device, float* target, uint32_t length, const uint32_t* indices,
                                      const float* deltas, const uint64_t* story_offsets, uint32_t stories,
                                      float lo, float hi, float* const* replicas, uint32_t replica_count,
                                      void* stream, uint32_t* updates);

/* Bytes of device scratch that leo_b200_sparse_mean_apply holds on `device`
   (0 before its first call there; the static variant never adds to it). */
size_t leo_b200_sparse_apply_scratch_bytes(int device);

#ifdef __cplusplus
}
#endif

#endif /* LEO_B200_H */
