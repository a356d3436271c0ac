// Launch geometry shared by every causal-softmax kernel and the host planner.
//
// Layout in HBM: `batch` matrices, matrix b starting at element
// b * batch_stride; each matrix is `rows` rows of `pitch` FP16 elements
// (pitch >= cols, pitch % 8 == 0, so every row starts 16-byte aligned).
// Local row i of a launch is absolute causal row (row_offset + i): it has
// valid = min(row_offset + i + 1, cols) probabilities, and every other
// column of the output row, padding included, is written +0.0 (0x0000).
#pragma once

#include <stdint.h>

namespace cs {

struct Geometry {
  const uint16_t* in;
  uint16_t* out;
  int64_t batch;
  int64_t batch_stride;  // elements between consecutive matrices
  int32_t rows;          // rows in this launch (a row block when sharded)
  int32_t cols;
  int32_t pitch;         // elements per row in memory
  int32_t row_offset;    // absolute causal row of local row 0
  float scale;
  uint32_t* status;      // device status word (atomicOr of kStatus* bits)
  uint32_t* sched;       // row-resident kernel: {claim, done} counters of the dynamic
                         // schedule, zero between launches; nullptr: static schedule
  uint64_t timeout_ns;   // bound on every mbarrier wait
  uint32_t flags;        // debug flags (kFlag*), 0 in production launches
};

// Work units of the row-resident kernels. Rows whose causal prefix is shorter
// than `cols` ("triangle rows", the first n_tri local rows) are paired
// (i, n_tri-1-i) so every pair carries the same number of elements,
// 2*row_offset + n_tri + 1; an odd middle row and the full-width rows
// (valid == cols) are single units.
struct UnitMap {
  int32_t n_tri;
  int32_t n_pairs;
  int32_t units_per_matrix;
  int64_t total_units;
};

__host__ __device__ __forceinline__ int32_t valid_cols(const Geometry& g, int32_t local_row) {
  const int64_t v = (int64_t)g.row_offset + local_row + 1;
  return v < g.cols ? (int32_t)v : g.cols;
}

// paired == false makes every row its own unit (used when a pair would not
// fit the kernel's registers but a single row does).
__host__ __device__ __forceinline__ UnitMap make_unit_map(const Geometry& g, bool paired = true) {
  UnitMap m;
  int64_t tri = (int64_t)g.cols - 1 - g.row_offset;  // rows with valid < cols
  if (tri < 0) tri = 0;
  if (tri > g.rows) tri = g.rows;
  if (!paired) tri = 0;
  m.n_tri = (int32_t)tri;
  m.n_pairs = m.n_tri / 2;
  m.units_per_matrix = m.n_pairs + (m.n_tri & 1) + (g.rows - m.n_tri);
  m.total_units = (int64_t)m.units_per_matrix * g.batch;
  return m;
}

// Unit k of a matrix -> (row_a, row_b); row_b < 0 for a single-row unit.
__host__ __device__ __forceinline__ void unit_rows(const UnitMap& m, int32_t k, int32_t& row_a,
                                                   int32_t& row_b) {
  if (k < m.n_pairs) {
    row_a = k;
    row_b = m.n_tri - 1 - k;
    return;
  }
  const int32_t j = k - m.n_pairs;
  row_b = -1;
  if (m.n_tri & 1)
    row_a = (j == 0) ? m.n_pairs : m.n_tri + j - 1;
  else
    row_a = m.n_tri + j;
}

}  // namespace cs
