// tile_sched.h -- linear tile id -> (m_tile, n_tile) for the persistent GEMM kernels.
//
// Same rasterization as the reference (src/gemm_bench.cu:231-252): tiles are numbered
// row-major over a tiles_m x tiles_n grid; with group > 1 the grid is cut into bands of
// `group` M-tiles and each band is walked column-major, so the tiles that run at the same
// time share B panels (N x K) and a few A panels in L2. A persistent CTA visits linear ids
// blockIdx.x, blockIdx.x + gridDim.x, ...; one wave of 148 SMs therefore covers about
// 148 / group columns of one band.
#pragma once

#if defined(__CUDACC__)
#define B2G_HD __host__ __device__ __forceinline__
#else
#define B2G_HD inline
#endif

namespace b2g {

B2G_HD void tile_coord(int linear, int tiles_m, int tiles_n, int group, int& m_tile,
                       int& n_tile) {
    if (group <= 1) {
        m_tile = linear / tiles_n;
        n_tile = linear - m_tile * tiles_n;
        return;
    }
    const int band = linear / (group * tiles_n);
    const int first = band * group;
    const int rows = (tiles_m - first) < group ? (tiles_m - first) : group;
    const int idx = linear - first * tiles_n;
    m_tile = first + idx % rows;
    n_tile = idx / rows;
}

}  // namespace b2g
