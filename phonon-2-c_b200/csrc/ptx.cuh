// ptx.cuh - thin inline-PTX wrappers for sm_100a: mbarriers with bounded waits, TMA tile loads, tcgen05 (TMEM
// allocation, int8 MMA, commit, loads) and the shared-memory matrix descriptors the MMA reads its operands through.
//
// Every wait is bounded: a wait that runs out sets the launch's error word and the kernel's abort flag and returns
// false, so a kernel never spins forever on a barrier that will not complete.
#pragma once
#include <cstdint>
#include <cuda.h>

namespace p2cu {

// Device-side error codes written to the launch's error word (first error wins).
enum : uint32_t { DEV_OK = 0, DEV_TIMEOUT_FULL = 1, DEV_TIMEOUT_READY = 2, DEV_TIMEOUT_EMPTY = 3,
                  DEV_TIMEOUT_ACC = 4, DEV_TIMEOUT_DRAIN = 5, DEV_BAD_ARGS = 6 };

// About one to two seconds of polling on a B200 before a wait gives up.
constexpr uint32_t WAIT_LIMIT = 1u << 25;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarriers ---------------------------------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}

// Non-blocking test of the phase (acquire on success). On a phase that has already completed it returns at once,
// where try_wait was measured at about 90 ns per call on B200 - a cost a single MMA-issuing thread pays per barrier
// (two waits per K stage slowed a stage's issue by 0.19 us).
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}

// Wait for the phase of `bar` with the given parity to complete: a test first, then try_wait polls (which let the
// hardware suspend the thread between polls). Returns false (after recording `code` in *err and setting *abort) when
// `limit` polls run out or another role already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t code,
                                          uint32_t* err, volatile int* abort_flag, uint32_t limit = WAIT_LIMIT) {
    const uint32_t a = smem_u32(bar);
    if (mbar_test_wait(a, parity)) return true;
    for (uint32_t i = 0; i < limit; ++i) {
        if (mbar_try_wait(a, parity)) return true;
        if ((i & 1023u) == 1023u && *abort_flag) return false;
    }
    if (err) atomicCAS(err, DEV_OK, code);
    *abort_flag = 1;
    return false;
}

// The same wait with a pause between polls, for waits expected to last microseconds (an epilogue waiting for the
// last MMA, a producer draining its copies), so that a tight poll loop does not take issue slots from the warps
// doing the work. About the same bound in time as mbar_wait.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t code, uint32_t* err,
                                                volatile int* abort_flag) {
    const uint32_t a = smem_u32(bar);
    for (uint32_t i = 0; i < (WAIT_LIMIT >> 5); ++i) {
        if (mbar_test_wait(a, parity)) return true;
        if (*abort_flag) return false;
        __nanosleep(64);
    }
    if (err) atomicCAS(err, DEV_OK, code);
    *abort_flag = 1;
    return false;
}

// Wait for a barrier phase with one polling lane per warp; every lane then acquires the completed phase. The whole
// warp must call it; every lane gets the same result.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, uint32_t code, uint32_t* err,
                                          volatile int* abort_flag, bool sleep = false) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0)
        ok = (sleep ? mbar_wait_sleep(bar, parity, code, err, abort_flag)
                    : mbar_wait(bar, parity, code, err, abort_flag)) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok) mbar_test_wait(smem_u32(bar), parity);   // already complete: acquire for this lane
    return ok != 0;
}

// The same wait for a converged warp whose lanes all poll at once (no lane waits alone, so no branch leaves the warp
// diverged): every lane sees the same phase and returns the same result. For loops that one elected lane's issue
// follows (the MMA issuers): issue from code that one lane runs alone, with branches inside it, was measured at about
// half the rate of the same instructions in a converged warp.
__device__ __forceinline__ bool warp_wait_all(uint64_t* bar, uint32_t parity, uint32_t code, uint32_t* err,
                                              volatile int* abort_flag, uint32_t limit = WAIT_LIMIT) {
    const uint32_t a = smem_u32(bar);
    if (mbar_test_wait(a, parity)) return true;
    for (uint32_t i = 0; i < limit; ++i) {
        if (mbar_try_wait(a, parity)) return true;
        if ((i & 1023u) == 1023u && *abort_flag) return false;
    }
    if (err && (threadIdx.x & 31) == 0) atomicCAS(err, DEV_OK, code);
    *abort_flag = 1;
    return false;
}

// One lane of a converged warp: 1 in the elected lane, 0 in the others.
__device__ __forceinline__ uint32_t elect_one() {
    uint32_t e;
    asm volatile("{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}" : "=r"(e));
    return e;
}

// ---- TMA ---------------------------------------------------------------------------------------------------------

// Prefetch the 128-byte line holding `p` into L2. L2 is where every SM's accesses meet, so a prefetch issued before a
// dependency wait cannot hand out stale data: a later write by the kernel waited for updates the line there.
__device__ __forceinline__ void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" :: "l"(p) : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load of one box into this CTA's shared memory whose completion is signalled on `bar_cluster`, an mbarrier
// of either CTA of a CTA pair (a shared::cluster address, e.g. the even CTA's from cluster_map). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster,
                                                 int32_t x, int32_t y) {
    asm volatile("cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4}], [%2];"
                 :: "r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster),
                    "r"(x), "r"(y) : "memory");
}

// 2-D tiled load of one box into shared memory, completing `bytes` of transaction on `bar`. No multicast.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4}], [%2];"
                 :: "r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)),
                    "r"(x), "r"(y) : "memory");
}

// 2-D tiled store of one box from shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int32_t x, int32_t y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 :: "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(smem_src)), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void tma_store_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until every committed bulk store of this thread has completed (its writes performed).
__device__ __forceinline__ void tma_store_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Wait until every committed bulk store of this thread has finished reading its shared-memory source.
__device__ __forceinline__ void tma_store_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// The same for all but the most recently committed store.
__device__ __forceinline__ void tma_store_wait_read_1() {
    asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

// Programmatic dependent launch: let the next kernel in the stream begin, and wait for the previous ones' writes.
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Barrier among `count` threads (a multiple of 32) of the CTA, id 1..15 (0 is __syncthreads).
__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t count) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(count) : "memory");
}

// Generic-proxy writes to shared memory made visible to the async proxy (the tensor cores read operands there).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- tcgen05 -----------------------------------------------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {   // whole warp
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {                                  // whole warp
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {       // whole warp
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem], int8 x int8 -> int32, one CTA. `accumulate` = 0 overwrites D.
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}

// D[tmem] (+)= A[smem] * B[smem], tf32 x tf32 -> fp32 (the low 13 mantissa bits of each operand are ignored).
__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(bar)) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane (base lane + i), columns col..col+31.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                   "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
                   "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
}
// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15])
                 : "r"(taddr));
}
// 32 lanes x 8 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// Thread i of the warp writes lane (base lane + i), columns col..col+7.
__device__ __forceinline__ void tmem_st_32x32b_x8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
                 :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
                    "r"(r[7]) : "memory");
}
// This thread's tcgen05.st writes have completed.
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// D[tmem] (+)= A[tmem] * B[smem], int8 x int8 -> int32, one CTA: A (M = 128 rows, one per TMEM lane, four 8-bit K
// values per 32-bit column, K-major) is read from tensor memory at tmem_a.
__device__ __forceinline__ void mma_i8_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}"
                 :: "r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}

// The same MMA and commit issued by the lane whose `lead` is non-zero, the whole warp executing them (a predicate,
// not a branch, selects the lane).
__device__ __forceinline__ void mma_i8_ts_lead(uint32_t lead, uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                               uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred e, p;\n\t"
                 "setp.ne.b32 e, %5, 0;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}"
                 :: "r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(lead) : "memory");
}
__device__ __forceinline__ void mma_i8_lead(uint32_t lead, uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred e, p;\n\t"
                 "setp.ne.b32 e, %5, 0;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(lead) : "memory");
}
__device__ __forceinline__ void mma_tf32_lead(uint32_t lead, uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred e, p;\n\t"
                 "setp.ne.b32 e, %5, 0;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(lead) : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem], tf32 x tf32 -> fp32: A (M = 128 rows, one per TMEM lane, one tf32 K value per
// 32-bit column) read from tensor memory at tmem_a.
__device__ __forceinline__ void mma_tf32_ts_lead(uint32_t lead, uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                                 uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred e, p;\n\t"
                 "setp.ne.b32 e, %5, 0;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}"
                 :: "r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(lead) : "memory");
}
__device__ __forceinline__ void mma_commit_lead(uint32_t lead, uint64_t* bar) {
    asm volatile("{\n\t.reg .pred e;\n\t"
                 "setp.ne.b32 e, %1, 0;\n\t"
                 "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}"
                 :: "r"(smem_u32(bar)), "r"(lead) : "memory");
}

// ---- CTA pairs (clusters of two, tcgen05 cta_group::2) ------------------------------------------------------------

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// The shared::cluster address of the object at the same offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_map(const void* local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
    return r;
}
// Arrive (release at cluster scope) on an mbarrier of another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" :: "r"(cluster_addr) : "memory");
}
// Arrive without ordering on an mbarrier of another CTA of the cluster: for signals whose payload the signalling
// thread has only observed (a TMA completion it waited for), not written.
__device__ __forceinline__ void mbar_arrive_remote_relaxed(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" :: "r"(cluster_addr) : "memory");
}
// Every thread of both CTAs: a full cluster barrier (release / acquire).
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {   // the same warp in both CTAs
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}
// D[tmem of both CTAs] (+)= A[smem of both CTAs, M = 256] * B[N split between the CTAs]; issued by the even CTA.
__device__ __forceinline__ void mma_i8_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
// Arrive on the mbarrier at `bar`'s offset in every CTA of `cta_mask` once this thread's pair MMAs have completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 :: "r"(smem_u32(bar)), "h"(cta_mask) : "memory");
}

// The pair MMA and its commit from the lane whose `lead` is non-zero, the whole warp executing them.
__device__ __forceinline__ void mma_i8_pair_lead(uint32_t lead, uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                                 uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred e, p;\n\t"
                 "setp.ne.b32 e, %5, 0;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "@e tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(lead) : "memory");
}
__device__ __forceinline__ void mma_commit_pair_lead(uint32_t lead, uint64_t* bar, uint16_t cta_mask) {
    asm volatile("{\n\t.reg .pred e;\n\t"
                 "setp.ne.b32 e, %2, 0;\n\t"
                 "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}"
                 :: "r"(smem_u32(bar)), "h"(cta_mask), "r"(lead) : "memory");
}

// ---- descriptors ---------------------------------------------------------------------------------------------------

// Shared-memory matrix descriptor (tcgen05): start address, leading / stride byte offsets (all >> 4), version 1,
// base offset 0, and the swizzle mode in bits 61-63 (2 = 128-byte swizzle, 4 = 64-byte, 6 = 32-byte, 0 = none).
enum : uint32_t { SWZ_NONE = 0, SWZ_128B = 2, SWZ_64B = 4, SWZ_32B = 6 };

__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t swizzle) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;                       // descriptor version for sm_100
    d |= static_cast<uint64_t>(swizzle & 7u) << 61;
    return d;
}

// Instruction descriptor for kind::i8 with signed A and B, int32 accumulators. a_mn / b_mn select MN-major operands.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N, bool a_mn, bool b_mn) {
    return (2u << 4)                                  // D format: s32
         | (1u << 7)                                  // A: signed 8-bit
         | (1u << 10)                                 // B: signed 8-bit
         | ((a_mn ? 1u : 0u) << 15)
         | ((b_mn ? 1u : 0u) << 16)
         | (static_cast<uint32_t>(N >> 3) << 17)
         | (static_cast<uint32_t>(M >> 4) << 24);
}

// Instruction descriptor for kind::tf32 with fp32 accumulators; A K-major, B K-major or (b_mn) MN-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N, bool b_mn) {
    return (1u << 4)                                  // D format: f32
         | (2u << 7)                                  // A: tf32
         | (2u << 10)                                 // B: tf32
         | ((b_mn ? 1u : 0u) << 16)
         | (static_cast<uint32_t>(N >> 3) << 17)
         | (static_cast<uint32_t>(M >> 4) << 24);
}

}  // namespace p2cu
