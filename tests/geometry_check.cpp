// Brute-force check of the launch geometry (kernels/geometry.cuh) on the CPU.
// The header's __host__ __device__ functions are compiled here as plain C++
// (the test defines the CUDA qualifiers away), so this checks the very code
// the kernels and the planner run.
//
// stdin: one geometry per line, "rows cols row_offset split_row split_shift".
// stdout, per geometry: "n_tri units bound max_vectors min_pair max_pair ok"
//   bound        unit_max_vectors(), the stage size the planner allocates
//   max_vectors  the largest unit actually mapped (16-byte vectors)
//   min/max_pair least / most causal elements of a row pair (0 0 if none)
//   ok           1 if every local row is in exactly one unit (paired and
//                single-row maps), the triangle rows are exactly the first
//                n_tri rows, and no unit exceeds the bound
#include <cstdint>
#include <cstdio>
#include <vector>

#include "geometry.cuh"

int main() {
  long long rows, cols, off, split, shift;
  while (std::scanf("%lld %lld %lld %lld %lld", &rows, &cols, &off, &split, &shift) == 5) {
    cs::Geometry g{};
    g.batch = 1;
    g.rows = (int32_t)rows;
    g.cols = (int32_t)cols;
    g.pitch = (int32_t)((cols + 7) / 8 * 8);
    g.row_offset = (int32_t)off;
    g.split_row = (int32_t)split;
    g.split_shift = (int32_t)shift;
    bool ok = true;
    int64_t max_nv = 0, min_pair = 0, max_pair = 0, n_tri = 0, units = 0, bound = 0;
    for (int paired = 1; paired >= 0; --paired) {
      const cs::UnitMap m = cs::make_unit_map(g, paired != 0);
      const int64_t b = cs::unit_max_vectors(g, m);
      std::vector<int> seen((size_t)rows, 0);
      for (int32_t k = 0; k < m.units_per_matrix; ++k) {
        int32_t ra = -1, rb = -1;
        cs::unit_rows(m, k, ra, rb);
        if (ra < 0 || ra >= rows || rb >= rows) {
          ok = false;
          break;
        }
        ++seen[(size_t)ra];
        const int64_t va = cs::valid_cols(g, ra);
        int64_t nv = (va + 7) / 8;
        if (rb >= 0) {
          ++seen[(size_t)rb];
          const int64_t vb = cs::valid_cols(g, rb);
          nv += (vb + 7) / 8;
          if (paired) {
            const int64_t s = va + vb;
            if (min_pair == 0 || s < min_pair) min_pair = s;
            if (s > max_pair) max_pair = s;
          }
        }
        if (nv > b) ok = false;
        if (paired && nv > max_nv) max_nv = nv;
      }
      for (long long r = 0; r < rows; ++r)
        if (seen[(size_t)r] != 1) ok = false;
      if (paired) {
        n_tri = m.n_tri;
        units = m.units_per_matrix;
        bound = b;
        for (long long r = 0; r < rows; ++r)
          if ((cs::valid_cols(g, (int32_t)r) < cols) != (r < m.n_tri)) ok = false;
      }
    }
    std::printf("%lld %lld %lld %lld %lld %lld %d\n", (long long)n_tri, (long long)units, (long long)bound,
                (long long)max_nv, (long long)min_pair, (long long)max_pair, ok ? 1 : 0);
  }
  return 0;
}
