// Device helpers shared by the Fry kernels: mbarriers with bounded waits, TMA tile loads,
// tcgen05 (TMEM allocation, MMA issue, commit, loads), and the library's error flag.
// sm_100a only. No TMA load here uses cluster multicast: the same code runs on every GPU of a box.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <map>
#include <tuple>
#include <utility>

#define FRY_DEVICE __device__ __forceinline__

namespace fry {

// Error codes a kernel records in the device-side status word (first failure wins).
enum DeviceError : int {
    kOk = 0,
    kWaitTimeout = 1,      // a bounded mbarrier wait gave up
    kBadToken = 2,         // a board token outside the vocabulary
    kBadShape = 3,         // a launch got a shape its kernel does not take
    kMisaligned = 4,       // dynamic shared memory did not start on the 1024-byte boundary a kernel lays out from
    kBadColumn = 5,        // a lean lane's answer column outside the answer row
    kNotPositiveDefinite = 6,  // a GPTQ Cholesky factorization met a pivot that is not positive (where: the column)
};

// Set by kernels on a failure they can detect; read and cleared by fry_device_status(). The library is one
// translation unit (fry_b200.cu includes every kernel file), so this is its only definition.
__device__ int g_status[2];  // [code, where]

FRY_DEVICE void record_error(int code, int where) {
    if (atomicCAS(&g_status[0], 0, code) == 0) g_status[1] = where;
}

// Time bound for every wait on an mbarrier, in ns of the global timer: by default 2 s, far beyond any real wait
// (microseconds). fry_set_wait_limit_ns changes it per device; a kernel reads it when a wait first spins.
constexpr uint64_t kDefaultWaitLimitNs = 2000000000ull;
__device__ uint64_t g_wait_limit_ns = kDefaultWaitLimitNs;

FRY_DEVICE uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

FRY_DEVICE uint32_t smem_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

FRY_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

FRY_DEVICE void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

FRY_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

FRY_DEVICE void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

FRY_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Waits for the phase of the given parity to complete; false (and the error flag set) if it never does.
FRY_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, int where) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = global_timer_ns(), limit = g_wait_limit_ns;
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0 && global_timer_ns() - start > limit) break;
    }
    record_error(kWaitTimeout, where);
    return false;
}

// ---- thread-block clusters: distributed shared memory and remote mbarrier arrivals ----
FRY_DEVICE uint32_t cluster_rank() {
    uint32_t rank;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    return rank;
}
// The address of `p` (this CTA's shared memory) in the shared memory of cluster CTA `rank`.
FRY_DEVICE uint32_t peer_smem(const void* p, uint32_t rank) {
    uint32_t address;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(address) : "r"(smem_addr(p)), "r"(rank));
    return address;
}
FRY_DEVICE void st_peer_f32x2(uint32_t address, float a, float b) {
    asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(address), "f"(a), "f"(b) : "memory");
}
// An arrival on a cluster CTA's mbarrier, releasing this thread's earlier writes (its st.shared::cluster among them).
FRY_DEVICE void mbar_arrive_peer(uint32_t address) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(address) : "memory");
}
// An arrival on a cluster CTA's mbarrier that publishes no memory of its own (release at CTA scope, the instruction's
// default): a hand-over whose ordering other fences provide, such as TMEM reads before tcgen05's thread-sync fence.
FRY_DEVICE void mbar_arrive_remote(uint32_t address) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(address) : "memory");
}
FRY_DEVICE bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
// mbar_wait for a barrier that other CTAs of the cluster arrive on (acquiring their writes), bounded the same way.
FRY_DEVICE bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int where) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t start = global_timer_ns(), limit = g_wait_limit_ns;
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((i & 255u) == 0 && global_timer_ns() - start > limit) break;
    }
    record_error(kWaitTimeout, where);
    return false;
}
// Every thread of every CTA of the cluster (all threads reach it: it does not wait for ever only if they do).
FRY_DEVICE void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// 2-D tiled TMA load of box {x, y} (x the contiguous coordinate) into shared memory, completing on bar.
FRY_DEVICE void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y)
        : "memory");
}

// 2-D tiled TMA store of box {x, y} from shared memory, in this thread's current bulk async-group.
FRY_DEVICE void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
                 "r"(smem_addr(src)), "r"(x), "r"(y)
                 : "memory");
}
FRY_DEVICE void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// every bulk async-group of this thread has finished reading its shared memory
FRY_DEVICE void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// waits until at most N of this thread's committed bulk groups have not yet read their shared-memory sources
template <int N>
FRY_DEVICE void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// every bulk async-group of this thread has completed
FRY_DEVICE void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// 16 bytes global -> shared without a register round trip (L2 only), in this thread's current cp.async group
FRY_DEVICE void cp_async16(void* shared, const void* global) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(shared))), "l"(global)
                 : "memory");
}
FRY_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// waits until at most PENDING of this thread's cp.async groups are still in flight
template <int PENDING>
FRY_DEVICE void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(PENDING) : "memory"); }
// orders this thread's shared-memory accesses before later async-proxy (TMA) accesses
FRY_DEVICE void fence_proxy_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

FRY_DEVICE void prefetch_tensor_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

FRY_DEVICE bool elect_one() {
    uint32_t pred;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "elect.sync _|p, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// ---- tcgen05 -------------------------------------------------------------------------------------------

FRY_DEVICE void tmem_alloc(uint32_t* dst_smem, uint32_t columns) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)), "r"(columns)
                 : "memory");
}
FRY_DEVICE void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
FRY_DEVICE void tmem_dealloc(uint32_t addr, uint32_t columns) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(addr), "r"(columns) : "memory");
}
FRY_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
FRY_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T for one MMA instruction; kind::i8 or kind::f16 by template.
template <int KIND>
FRY_DEVICE void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    if constexpr (KIND == 0) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
    }
}

// Arrives on bar once every MMA this thread issued before it has completed.
FRY_DEVICE void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// ---- CTA pairs (cta_group::2): one MMA of M = 256 rows whose A halves and B halves lie in the shared memory of the two
// CTAs of a cluster, at the same offsets, and whose accumulator halves lie in each CTA's TMEM (rows 0-127 in the even
// CTA's, 128-255 in the odd one's). The even CTA issues the MMAs; every tcgen05 instruction of such a kernel is of the
// pair group. The TMEM allocation is one for the pair: a warp of each CTA allocates (and frees) it together.
FRY_DEVICE void tmem_alloc_pair(uint32_t* dst_smem, uint32_t columns) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)), "r"(columns)
                 : "memory");
}
FRY_DEVICE void tmem_relinquish_pair() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory"); }
FRY_DEVICE void tmem_dealloc_pair(uint32_t addr, uint32_t columns) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(addr), "r"(columns) : "memory");
}
template <int KIND>
FRY_DEVICE void mma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    if constexpr (KIND == 0) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
    }
}
// Arrives on the mbarrier at shared::cluster address `bar` (this CTA's or the peer's) once every pair MMA this thread
// issued before it has completed.
FRY_DEVICE void mma_commit_pair(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// 2-D tiled TMA load into this CTA's shared memory that completes on an mbarrier of either CTA of the pair (`bar` a
// shared::cluster address): both CTAs' operand loads complete on the even CTA's stage barrier. Each CTA loads only
// into its own shared memory.
FRY_DEVICE void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

// 32 consecutive 32-bit TMEM columns of this thread's lane (32x32b shape: lane i of the warp reads TMEM lane base+i).
FRY_DEVICE void tmem_load32(uint32_t addr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(addr));
}
FRY_DEVICE void tmem_load16(uint32_t addr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(addr));
}
FRY_DEVICE void tmem_load_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand tile in the 128-byte swizzle layout TMA writes:
// rows of 128 bytes, 8-row (1024-byte) swizzle atoms stacked along M/N. Fields: start address >> 4 [0,14),
// leading byte offset >> 4 [16,30) (unused for swizzled K-major, set to 1), stride byte offset >> 4 [32,46)
// (1024 bytes between 8-row groups), descriptor version 1 [46,48), swizzle mode 2 = 128B [61,64).
FRY_DEVICE uint64_t smem_desc_sw128(uint32_t smem_byte_addr) {
    uint64_t desc = 0;
    desc |= static_cast<uint64_t>((smem_byte_addr >> 4) & 0x3FFF);
    desc |= static_cast<uint64_t>(1) << 16;
    desc |= static_cast<uint64_t>(1024 >> 4) << 32;
    desc |= static_cast<uint64_t>(1) << 46;
    desc |= static_cast<uint64_t>(2) << 61;
    return desc;
}

// Instruction descriptor for a dense MMA with both operands K-major, M = 128 rows (256 for a CTA pair's):
// D format [4,6) (1 f32, 2 s32), A format [7,10) and B format [10,13) (kind::i8: 1 signed; kind::f16: 0 f16),
// N >> 3 at [17,23), M >> 4 at [24,29).
template <int KIND>
__host__ __device__ constexpr uint32_t instr_desc(int n, int m = 128) {
    return (KIND == 0 ? (2u << 4) | (1u << 7) | (1u << 10) : (1u << 4)) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

// ---- programmatic dependent launch ---------------------------------------------------------------------
//
// Every kernel of the library is launched with programmatic stream serialization, so it may start (launch, take its
// shared memory, set up) while the kernel before it in the stream finishes. Each kernel calls grid_dependency_start()
// before it reads or writes anything an earlier kernel touches, in every CTA: that waits until the previous grid has
// completed with its memory visible, so a kernel's completion still implies every earlier one's, then lets the next
// kernel be scheduled.
FRY_DEVICE void grid_dependency_start() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... Params, typename... Args>
inline cudaError_t launch_dependent(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t config = {};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    return cudaLaunchKernelEx(&config, kernel, static_cast<Params>(args)...);
}

// launch_dependent in thread-block clusters of `cluster` CTAs along x (grid.x a multiple of it).
template <typename... Params, typename... Args>
inline cudaError_t launch_dependent_cluster(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, int cluster, cudaStream_t stream,
                                            Args... args) {
    cudaLaunchConfig_t config = {};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    cudaLaunchAttribute attribute[2];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    attribute[1].id = cudaLaunchAttributeClusterDimension;
    attribute[1].val.clusterDim.x = static_cast<unsigned>(cluster);
    attribute[1].val.clusterDim.y = 1;
    attribute[1].val.clusterDim.z = 1;
    config.attrs = attribute;
    config.numAttrs = 2;
    return cudaLaunchKernelEx(&config, kernel, static_cast<Params>(args)...);
}

// How many clusters of `cluster` CTAs of the kernel (with this block and shared memory) the device holds at once. The
// answer is kept per (kernel, device, shared memory, cluster): the occupancy query costs host time on every launch
// otherwise, which eager (ungraphed) forwards pay per GEMM.
template <typename... Params>
inline cudaError_t max_active_clusters(void (*kernel)(Params...), dim3 block, size_t smem, int cluster, int* count) {
    static std::mutex mutex;
    static std::map<std::tuple<const void*, int, size_t, int, unsigned>, int> known;
    int device = 0;
    const cudaError_t found_device = cudaGetDevice(&device);
    if (found_device != cudaSuccess) return found_device;
    const auto key = std::make_tuple(reinterpret_cast<const void*>(kernel), device, smem, cluster, block.x * block.y * block.z);
    {
        std::lock_guard<std::mutex> lock(mutex);
        const auto found = known.find(key);
        if (found != known.end()) {
            *count = found->second;
            return cudaSuccess;
        }
    }
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(cluster);
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeClusterDimension;
    attribute[0].val.clusterDim.x = static_cast<unsigned>(cluster);
    attribute[0].val.clusterDim.y = 1;
    attribute[0].val.clusterDim.z = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    const cudaError_t status = cudaOccupancyMaxActiveClusters(count, reinterpret_cast<const void*>(kernel), &config);
    if (status == cudaSuccess) {
        std::lock_guard<std::mutex> lock(mutex);
        known[key] = *count;
    }
    return status;
}

// ---- small numeric helpers -----------------------------------------------------------------------------

// Two fp32 lanes in one 64-bit register, for the paired (f32x2) IEEE adds, multiplies and FMAs of sm_100: each lane
// rounds exactly as the scalar instruction does.
FRY_DEVICE uint64_t pair2(float lo, float hi) {
    uint64_t v;
    asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(lo), "f"(hi));
    return v;
}
FRY_DEVICE float2 lanes(uint64_t v) {
    float2 f;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(f.x), "=f"(f.y) : "l"(v));
    return f;
}
FRY_DEVICE uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
FRY_DEVICE uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
FRY_DEVICE uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

FRY_DEVICE float ex2_approx(float x) {
    float y;
    asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// 2^x with denormal results flushed to zero (the bare 2^x instruction): where 2^x only enters 1 + 2^x or a softmax's
// probabilities, which fp16 rounds to 0 far above fp32's denormals, the results are those of ex2_approx
FRY_DEVICE float ex2_approx_ftz(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// 1/x by the reciprocal instruction alone (at most 1 ulp off; no full-range scaling: for x from 1 up, where it is exact
// in range and gives 0 at infinity)
FRY_DEVICE float rcp_approx_ftz(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
FRY_DEVICE float div_full(float a, float b) {
    float y;
    asm("div.full.f32 %0, %1, %2;" : "=f"(y) : "f"(a), "f"(b));
    return y;
}
FRY_DEVICE float warp_sum(float v) {
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
    return v;
}
FRY_DEVICE float warp_max(float v) {
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, s));
    return v;
}
// The warp's maximum of v in one instruction (sm_100's f32 redux.sync); NaN lanes are ignored, as fmaxf ignores them.
FRY_DEVICE float warp_max_redux(float v) {
    float m;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(m) : "f"(v));
    return m;
}
// fp16 -> fp32 on the FMA pipe rather than the conversion unit (a quarter of its rate or less): the mixed-precision add
// (PTX add.f32.f16, sm_100) of -0.0, exact for every finite or infinite input (a NaN stays a NaN).
FRY_DEVICE float h2f_exact(uint16_t bits) {
    float value;
    asm("add.rn.f32.f16 %0, %1, %2;" : "=f"(value) : "h"(bits), "f"(-0.0f));
    return value;
}
// Two fp32 values rounded to fp16 and packed (lo in the low half) by one conversion instruction.
FRY_DEVICE uint32_t pack_half2_rn(float lo, float hi) {
    const __half2 pair = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&pair);
}
// two fp32 values rounded to nearest-even bf16 in one instruction, lo in the low half
FRY_DEVICE uint32_t pack_bf162_rn(float lo, float hi) {
    uint32_t pair;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(pair) : "f"(hi), "f"(lo));
    return pair;
}
FRY_DEVICE float h2f(__half h) { return __half2float(h); }
FRY_DEVICE float h2f_bits(uint16_t bits) { return __half2float(__ushort_as_half(bits)); }
FRY_DEVICE uint16_t f2h_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }

// Raises a kernel's dynamic shared memory limit on the current device to at least `bytes` (it is never lowered, so
// launches of other sizes keep working); safe from several host threads.
inline cudaError_t ensure_smem(const void* kernel, int bytes) {
    static std::mutex mutex;
    static std::map<std::pair<const void*, int>, int> raised;
    int device = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status != cudaSuccess) return status;
    if (bytes <= 48 * 1024) return cudaSuccess;
    std::lock_guard<std::mutex> lock(mutex);
    int& current = raised[{kernel, device}];
    if (bytes <= current) return cudaSuccess;
    status = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (status == cudaSuccess) current = bytes;
    return status;
}

}  // namespace fry
