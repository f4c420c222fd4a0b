// Internal interface of the batch-end sparse mean apply (leo_sparse_apply.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#define LEO_SPARSE_APPLY_TILE 4096u        // tensor indices per merge tile (FP64 sums in shared memory)
#define LEO_SPARSE_APPLY_MAX_STORIES 256u  // stories per call (offsets travel as a kernel parameter)
#define LEO_SPARSE_APPLY_MAX_REPLICAS 64u  // replicas per call (pointers travel as a kernel parameter)
#define LEO_SPARSE_APPLY_MAX_DEVICES 64
#define LEO_SPARSE_APPLY_COUNTERS 64u      // leading scratch words: [0] merged count, [1] error flags
#define LEO_SPARSE_APPLY_STATIC_WORDS 262144u  // fixed scratch of the allocation-free entry point: 1 MiB

#define LEO_SPARSE_APPLY_ERR_RANGE 1u
#define LEO_SPARSE_APPLY_ERR_ORDER 2u
#define LEO_SPARSE_APPLY_ERR_DELTA 4u
#define LEO_SPARSE_APPLY_ERR_MERGED 8u

struct SparseApplyOffsets {
    uint64_t v[LEO_SPARSE_APPLY_MAX_STORIES + 1];
};
struct SparseApplyReplicas {
    float* ptr[LEO_SPARSE_APPLY_MAX_REPLICAS];
};

struct SparseApplyArgs {
    float* target;
    const uint32_t* indices;
    const float* deltas;
    uint32_t* scratch;  // LEO_SPARSE_APPLY_COUNTERS counters, then the [stories][tiles + 1] tile table
    uint32_t length, stories, tiles, replica_count;
    float lo, hi;
    SparseApplyOffsets offsets;
    SparseApplyReplicas replicas;
};

// Scratch words one call needs: counters plus the tile table.
size_t leo_sparse_apply_scratch_words(uint32_t length, uint32_t stories);
// Validates host-side arguments and fills `a` (everything but a.scratch).
void leo_sparse_apply_prepare(SparseApplyArgs& a, float* target, uint32_t length, const uint32_t* indices,
                              const float* deltas, const uint64_t* story_offsets, uint32_t stories, float lo, float hi,
                              float* const* replicas, uint32_t replica_count);
// Clears the counters, runs both kernels on `stream`, waits, checks the error
// flags (throwing std::runtime_error) and returns the merged index count.
uint32_t leo_sparse_apply_run(SparseApplyArgs& a, cudaStream_t stream);
