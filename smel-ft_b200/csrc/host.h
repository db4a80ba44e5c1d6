// Host-side helpers shared by the smelb entry points: per-device status word and SM count, last-error text and
// TMA tensor-map encoding (cuTensorMapEncodeTiled resolved through the runtime, so nothing links libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace smelb {

// 4-byte device word the kernels record wait timeouts in (allocated once per device)
int* device_status(int dev);

// Instrumentation: number of kernels launched by the library, and optional CUDA-event timing of the GEMM launches.
void count_launch();
bool gemm_timing_enabled();
void gemm_timing_begin(cudaStream_t st);
void gemm_timing_end(cudaStream_t st);
int num_sms(int dev);

// 2-D tiled tensor map over a row-major matrix [rows][cols] of `elem_bytes`-sized elements with row pitch
// `row_bytes`. box = {box_cols, box_rows}. swizzle_bytes: 0 (none), 32, 64 or 128 (box_cols * elem_bytes equal to
// it).
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows,
                 uint64_t cols, uint64_t row_bytes, uint32_t box_cols, uint32_t box_rows, int swizzle_bytes);

// 3-D tiled tensor map: dims {d0 (contiguous), d1, d2} with byte strides {d1, d2} (any order in memory), box
// {b0, b1, b2} landing in shared memory as [b2][b1][b0]; swizzle over b0 * elem bytes as in make_tmap_2d.
int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, const uint64_t dims[3],
                 const uint64_t strides_bytes[2], const uint32_t box[3], int swizzle_bytes);

}  // namespace smelb
