// Launch geometry shared by every causal-softmax kernel and the host planner.
//
// Layout in HBM: `batch` matrices, matrix b starting at element
// b * batch_stride; each matrix is `rows` rows of `pitch` FP16 elements
// (pitch >= cols, pitch % 8 == 0, so every row starts 16-byte aligned).
// Local row i of a launch is absolute causal row row_offset + i, plus
// split_shift when i >= split_row: a folded launch holds a second row block,
// stored right after the first, that starts split_shift rows past the first
// one's end (split_row = split_shift = 0: one block).
// A row with absolute index a has valid = min(a + 1, cols) probabilities,
// and every other column of the output row, padding included, is written
// +0.0 (0x0000).
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
  int32_t split_row;     // first local row of the second row block (0: none)
  int32_t split_shift;   // rows skipped between the two blocks (>= 0)
  float scale;
  uint32_t* status;      // device status word (atomicOr of kStatus* bits)
  uint32_t* sched;       // row-resident kernel: {claim, done} counters of the dynamic
                         // schedule, zero between launches; nullptr: static schedule
  uint64_t timeout_ns;   // bound on every mbarrier wait
  uint32_t flags;        // debug flags (kFlag*), 0 in production launches
};

// Work units of the row-resident kernels. Rows whose causal prefix is shorter
// than `cols` ("triangle rows", the first n_tri local rows: absolute rows
// increase with the local row, also across a fold) are paired (i, n_tri-1-i)
// so every pair carries the same number of elements, 2*row_offset + n_tri + 1
// in one row block. In a folded launch the sum takes at most two values: one
// for pairs that take a row from each block and one for pairs within a
// block (for the mirror blocks [a, b) and [M-b, M-a) of an M x M matrix
// every pair crosses, and carries M + 1). An odd middle row and the
// full-width rows (valid == cols) are single units.
struct UnitMap {
  int32_t n_tri;
  int32_t n_pairs;
  int32_t units_per_matrix;
  int64_t total_units;
};

__host__ __device__ __forceinline__ int64_t abs_row(const Geometry& g, int32_t local_row) {
  return (int64_t)g.row_offset + local_row + (local_row >= g.split_row ? g.split_shift : 0);
}

__host__ __device__ __forceinline__ int32_t valid_cols(const Geometry& g, int32_t local_row) {
  const int64_t v = abs_row(g, local_row) + 1;
  return v < g.cols ? (int32_t)v : g.cols;
}

// Flat rows first, first + step, first + 2 step, ... of a launch (matrix b,
// row i), walked without a division per row: (b, i) advances by
// (step / rows, step % rows) with one carry. A flat row is inside the launch
// exactly when b < g.batch. The first row and the step are below 2^31 (a
// block or cluster index and the grid), so the set-up divides in 32 bits.
struct RowCursor {
  int64_t b;       // matrix
  int32_t i;       // row within the matrix
  int64_t step_b;  // step / rows
  int32_t step_i;  // step % rows
  __host__ __device__ __forceinline__ RowCursor(const Geometry& g, uint32_t first, uint32_t step) {
    const uint32_t rows = (uint32_t)g.rows;
    b = first / rows;
    i = (int32_t)(first - (uint32_t)b * rows);
    step_b = step / rows;
    step_i = (int32_t)(step - (uint32_t)step_b * rows);
  }
  __host__ __device__ __forceinline__ bool inside(const Geometry& g) const { return b < g.batch; }
  __host__ __device__ __forceinline__ void next(const Geometry& g) {
    b += step_b;
    // i and step_i are below rows < 2^31, so their sum fits 32 unsigned bits
    // (a signed sum would overflow once rows exceeds 2^31 - step).
    uint32_t n = (uint32_t)i + (uint32_t)step_i;
    if (n >= (uint32_t)g.rows) {
      n -= (uint32_t)g.rows;
      ++b;
    }
    i = (int32_t)n;
  }
  __host__ __device__ __forceinline__ int64_t offset(const Geometry& g) const {
    return b * g.batch_stride + (int64_t)i * g.pitch;
  }
};

// Rows of a block of n rows starting at absolute row first whose prefix is
// shorter than cols.
__host__ __device__ __forceinline__ int64_t block_triangle_rows(int64_t first, int64_t n, int64_t cols) {
  int64_t tri = cols - 1 - first;
  if (tri < 0) tri = 0;
  if (tri > n) tri = n;
  return tri;
}

__host__ __device__ __forceinline__ int64_t triangle_rows(const Geometry& g) {
  return block_triangle_rows(g.row_offset, g.split_row, g.cols) +
         block_triangle_rows((int64_t)g.row_offset + g.split_row + g.split_shift,
                             (int64_t)g.rows - g.split_row, g.cols);
}

// paired == false makes every row its own unit (used when a pair would not
// fit the kernel's registers but a single row does).
__host__ __device__ __forceinline__ UnitMap make_unit_map(const Geometry& g, bool paired = true) {
  UnitMap m;
  const int64_t tri = paired ? triangle_rows(g) : 0;  // rows with valid < cols
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

// Upper bound on the 16-byte vectors of one unit (what a stage must hold).
// A pair's element count is constant over each kind of pair (within one row
// block, or across a fold), and the pairs of one kind are contiguous in k
// from one end, so the first and the last pair bound them all; the +1
// covers the rounding of the pair's two rows.
__host__ __device__ __forceinline__ int64_t unit_max_vectors(const Geometry& g, const UnitMap& m) {
  int64_t mx = 0;
  for (int end = 0; end < 2 && m.n_pairs > 0; ++end) {
    const int32_t k = end ? m.n_pairs - 1 : 0;
    const int64_t nv = ((int64_t)valid_cols(g, k) + valid_cols(g, m.n_tri - 1 - k) + 7) / 8 + 1;
    if (nv > mx) mx = nv;
  }
  if (m.n_tri & 1) {
    const int64_t nv = ((int64_t)valid_cols(g, m.n_pairs) + 7) / 8;
    if (nv > mx) mx = nv;
  }
  if (g.rows > m.n_tri) {
    const int64_t nv = ((int64_t)g.cols + 7) / 8;
    if (nv > mx) mx = nv;
  }
  return mx;
}

}  // namespace cs
