// tcgen05 / TMEM TF32 GEMM for the 1x1 and implicit-GEMM convs.
// (Geometry planner and launcher; the kernel body is filled in by the
// tensor-core implementation.)
#pragma once

#include "k_simt.cuh"

namespace aie {

struct TcGeom {
    uint32_t bm, bn, split;
    uint64_t workspace_bytes;
    uint64_t grid;
};

static inline bool tc_available() { return false; }

static inline bool tc_igemm_supported(uint32_t, uint32_t, uint32_t, uint32_t, uint32_t) { return false; }

static inline int tc_plan(uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t,
                          uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, TcGeom *)
{
    return -1;
}

static inline int tc_launch(const TcGeom &, const ConvArgs &, void *, cudaStream_t, char *, size_t) { return -3; }

}  // namespace aie
