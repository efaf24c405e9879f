// dag.cuh -- device helpers of the moment-graph kernels (efs.cu k_dag and
// grad.cu k_dag_grad): mbarrier and bulk-copy primitives, 32-bit shared-memory
// accessors, record flag encoding and the block geometry.
#pragma once

#include "internal.hpp"

namespace mtpb {

__device__ __forceinline__ unsigned smem_u32(const void *p)
{
    return (unsigned)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(unsigned long long *bar, unsigned count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void bulk_load(void *dst, const void *src, unsigned bytes,
                                          unsigned long long *bar)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], "
                 "%2, [%3];" ::"r"(smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(unsigned long long *bar, unsigned parity)
{
    unsigned ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                 " selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(ok)
                 : "r"(smem_u32(bar)), "r"(parity)
                 : "memory");
    return ok != 0;
}

constexpr long DAG_WAIT_LIMIT = 1L << 22;   // bounded wait: sets the error flag

// Geometry: ATOMS atoms per block, two atoms per lane; a record stream is
// served by LPS = ATOMS/2 lanes, a warp serves SPW = 32/LPS streams and the
// block STREAMS streams.  Records are laid out warp-major per phase
// ([phase][warp][row][SPW streams], see dag_device_records) so that every warp
// streams its own contiguous records through a private double-buffered ring
// filled by TMA bulk copies: warps only meet at the phase barriers.
template <int ATOMS, int STREAMS> struct DagGeom {
    static constexpr int APT = 2;
    static constexpr int LPS = ATOMS / APT;
    static constexpr int SPW = 32 / LPS;
    static constexpr int WARPS = STREAMS / SPW;
    static constexpr int THREADS = WARPS * 32;
    static constexpr int CH = dag_chunk_rows(STREAMS);       // rows per ring slot
    static constexpr unsigned SLOT_BYTES = CH * SPW * sizeof(DagDevRec);
    static constexpr size_t ring_bytes() { return (size_t)WARPS * 2 * SLOT_BYTES; }
};

// shared-memory access with 32-bit addresses
__device__ __forceinline__ uint4 lds128(unsigned a)
{
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(a));
    return v;
}
__device__ __forceinline__ unsigned lds32(unsigned a)
{
    unsigned v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ double2 lds_d2(unsigned a)
{
    double2 v;
    asm volatile("ld.shared.v2.f64 {%0, %1}, [%2];" : "=d"(v.x), "=d"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts_d2(unsigned a, double x, double y)
{
    asm volatile("st.shared.v2.f64 [%0], {%1, %2};" ::"r"(a), "d"(x), "d"(y) : "memory");
}

// Row storage of the graph kernels: shared memory (32-bit addresses) or, for
// graphs larger than shared memory, a per-block slice of global scratch that
// stays resident in L2 (persistent blocks, one slice each).  Offsets are
// byte offsets from the lane's first atom in row 0.
template <bool GLOBAL_ROWS> struct Rows;
template <> struct Rows<false> {
    unsigned base;
    __device__ __forceinline__ double2 ld(unsigned off) const { return lds_d2(base + off); }
    __device__ __forceinline__ void st(unsigned off, double x, double y) const
    {
        sts_d2(base + off, x, y);
    }
};
template <> struct Rows<true> {
    char *base;
    __device__ __forceinline__ double2 ld(unsigned off) const
    {
        return *reinterpret_cast<const double2 *>(base + off);
    }
    __device__ __forceinline__ void st(unsigned off, double x, double y) const
    {
        *reinterpret_cast<double2 *>(base + off) = make_double2(x, y);
    }
};

constexpr unsigned DEV_END = 1u << 28, DEV_GLOBAL = 2u << 28, DEV_ENERGY = 4u << 28;
constexpr unsigned DEV_OUT_MASK = (1u << 28) - 1;

__device__ __forceinline__ void cp_async16(unsigned dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

} // namespace mtpb
