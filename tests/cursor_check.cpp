// Walk of the row cursor (kernels/geometry.cuh, RowCursor) on the CPU. The
// cursor is __host__ __device__ code; the test defines the CUDA qualifiers
// away and runs the very struct the online and cluster kernels use.
//
// stdin: one case per line, "rows batch step" (step = the launch's grid, or
// its cluster count). For each first row in {0, 1, step / 2, step - 1} below
// step, the cursor visits first, first + step, ... while it is inside the
// launch; every visit must equal (flat / rows, flat % rows), keep the row in
// [0, rows), and give the element offset b * batch_stride + i * pitch.
// stdout, per case: "visits ok".
#include <cstdint>
#include <cstdio>

#include "geometry.cuh"

int main() {
  long long rows, batch, step;
  while (std::scanf("%lld %lld %lld", &rows, &batch, &step) == 3) {
    cs::Geometry g{};
    g.batch = batch;
    g.rows = (int32_t)rows;
    g.cols = 8;
    g.pitch = 8;
    g.batch_stride = (int64_t)rows * 8;
    bool ok = true;
    long long visits = 0;
    const long long firsts[4] = {0, 1, step / 2, step - 1};
    for (int k = 0; k < 4 && ok; ++k) {
      const long long first = firsts[k];
      if (first < 0 || first >= step || (k > 0 && first == firsts[k - 1])) continue;
      cs::RowCursor cur(g, (uint32_t)first, (uint32_t)step);
      long long flat = first;
      for (; cur.inside(g); cur.next(g), flat += step) {
        ++visits;
        if (cur.b != flat / rows || cur.i != flat % rows || cur.i < 0 || cur.i >= rows ||
            cur.offset(g) != flat * 8) {
          ok = false;
          break;
        }
      }
      // The cursor leaves the launch exactly at the first flat row past it.
      if (ok && flat < rows * batch) ok = false;
    }
    std::printf("%lld %d\n", visits, ok ? 1 : 0);
  }
  return 0;
}
