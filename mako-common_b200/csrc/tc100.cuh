// sm_100a building blocks in inline PTX: mbarriers with bounded waits, TMA tensor loads, tcgen05 (UMMA, TMEM
// allocation, loads and stores, commit), and the shared-memory / instruction descriptors UMMA reads.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mako {
namespace tc {

// ---- mbarrier ------------------------------------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
// `count` arrivals at once (one thread standing for its warp after a __syncwarp).
__device__ __forceinline__ void mbar_arrive_n(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}\n"
                 : "=r"(ok)
                 : "r"(bar), "r"(parity)
                 : "memory");
    return ok != 0;
}
// As mbar_try_wait but never suspends the thread (mbarrier.test_wait): for loops that poll several barriers, where a
// suspended try_wait on one barrier would hold up work that another barrier has already released.
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}\n"
                 : "=r"(ok)
                 : "r"(bar), "r"(parity)
                 : "memory");
    return ok != 0;
}
// Waits for the phase of parity `parity` to complete; false when `limit` clock cycles pass first (the caller
// records the error and unwinds instead of spinning forever).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, long long limit)
{
    if (mbar_try_wait(bar, parity))
        return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > limit)
            return false;
    return true;
}

// ---- TMA -----------------------------------------------------------------------------------------------------------

// A 3-D tile of `map` at (c0, c1, c2) into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1, int c2)
{
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4, %5}], [%2];\n" ::"r"(dst),
                 "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}
// A 2-D box from this CTA's shared memory to global memory through `map` at (c0, c1), in the current bulk group
// (coordinates past the tensor's extent are not written).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int c0, int c1)
{
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];\n" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(src), "r"(c0), "r"(c1)
                 : "memory");
}
// `bytes` (a multiple of 16) from this CTA's shared memory to global memory, both addresses 16-byte aligned, in the
// current bulk group (untiled bulk copy: the copy engine does the global writes asynchronously).
__device__ __forceinline__ void bulk_store(void* gdst, uint32_t ssrc, uint32_t bytes)
{
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(gdst), "r"(ssrc), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
// Waits until every committed bulk copy of this thread has completed (its global writes included).
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }
// Waits until every committed bulk store has finished reading shared memory (the writes may still be in flight).
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map)
{
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- tcgen05 -------------------------------------------------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (fp16 or bf16 inputs, fp32 accumulate), issued by one thread.
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
                 "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
                 : "memory");
}
// As umma_ss with A read from tensor memory (row m in lane m, K along the columns, two 16-bit values a column).
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
                 "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
                 : "memory");
}
// `bar` receives one arrival when every tcgen05 operation this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
                 : "memory");
}

// 32 consecutive 32-bit columns of this thread's lane (warp-collective; the warp's lanes are 32 * (warp % 4) + lane).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                   "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
                   "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
}
// As tmem_ld32 for 64 or 128 consecutive columns in one instruction (r[c][e] = column 32 c + e): one TMEM read of a
// row's whole score tile instead of two or four.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[2][32])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n"
                 : "=r"(r[0][0]), "=r"(r[0][1]), "=r"(r[0][2]), "=r"(r[0][3]), "=r"(r[0][4]), "=r"(r[0][5]), "=r"(r[0][6]), "=r"(r[0][7]), "=r"(r[0][8]), "=r"(r[0][9]), "=r"(r[0][10]), "=r"(r[0][11]), "=r"(r[0][12]), "=r"(r[0][13]), "=r"(r[0][14]), "=r"(r[0][15]), "=r"(r[0][16]), "=r"(r[0][17]), "=r"(r[0][18]), "=r"(r[0][19]), "=r"(r[0][20]), "=r"(r[0][21]), "=r"(r[0][22]), "=r"(r[0][23]), "=r"(r[0][24]), "=r"(r[0][25]), "=r"(r[0][26]), "=r"(r[0][27]), "=r"(r[0][28]), "=r"(r[0][29]), "=r"(r[0][30]), "=r"(r[0][31]), "=r"(r[1][0]), "=r"(r[1][1]), "=r"(r[1][2]), "=r"(r[1][3]), "=r"(r[1][4]), "=r"(r[1][5]), "=r"(r[1][6]), "=r"(r[1][7]), "=r"(r[1][8]), "=r"(r[1][9]), "=r"(r[1][10]), "=r"(r[1][11]), "=r"(r[1][12]), "=r"(r[1][13]), "=r"(r[1][14]), "=r"(r[1][15]), "=r"(r[1][16]), "=r"(r[1][17]), "=r"(r[1][18]), "=r"(r[1][19]), "=r"(r[1][20]), "=r"(r[1][21]), "=r"(r[1][22]), "=r"(r[1][23]), "=r"(r[1][24]), "=r"(r[1][25]), "=r"(r[1][26]), "=r"(r[1][27]), "=r"(r[1][28]), "=r"(r[1][29]), "=r"(r[1][30]), "=r"(r[1][31])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, uint32_t (&r)[4][32])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95,%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,%112,%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127}, [%128];\n"
                 : "=r"(r[0][0]), "=r"(r[0][1]), "=r"(r[0][2]), "=r"(r[0][3]), "=r"(r[0][4]), "=r"(r[0][5]), "=r"(r[0][6]), "=r"(r[0][7]), "=r"(r[0][8]), "=r"(r[0][9]), "=r"(r[0][10]), "=r"(r[0][11]), "=r"(r[0][12]), "=r"(r[0][13]), "=r"(r[0][14]), "=r"(r[0][15]), "=r"(r[0][16]), "=r"(r[0][17]), "=r"(r[0][18]), "=r"(r[0][19]), "=r"(r[0][20]), "=r"(r[0][21]), "=r"(r[0][22]), "=r"(r[0][23]), "=r"(r[0][24]), "=r"(r[0][25]), "=r"(r[0][26]), "=r"(r[0][27]), "=r"(r[0][28]), "=r"(r[0][29]), "=r"(r[0][30]), "=r"(r[0][31]), "=r"(r[1][0]), "=r"(r[1][1]), "=r"(r[1][2]), "=r"(r[1][3]), "=r"(r[1][4]), "=r"(r[1][5]), "=r"(r[1][6]), "=r"(r[1][7]), "=r"(r[1][8]), "=r"(r[1][9]), "=r"(r[1][10]), "=r"(r[1][11]), "=r"(r[1][12]), "=r"(r[1][13]), "=r"(r[1][14]), "=r"(r[1][15]), "=r"(r[1][16]), "=r"(r[1][17]), "=r"(r[1][18]), "=r"(r[1][19]), "=r"(r[1][20]), "=r"(r[1][21]), "=r"(r[1][22]), "=r"(r[1][23]), "=r"(r[1][24]), "=r"(r[1][25]), "=r"(r[1][26]), "=r"(r[1][27]), "=r"(r[1][28]), "=r"(r[1][29]), "=r"(r[1][30]), "=r"(r[1][31]), "=r"(r[2][0]), "=r"(r[2][1]), "=r"(r[2][2]), "=r"(r[2][3]), "=r"(r[2][4]), "=r"(r[2][5]), "=r"(r[2][6]), "=r"(r[2][7]), "=r"(r[2][8]), "=r"(r[2][9]), "=r"(r[2][10]), "=r"(r[2][11]), "=r"(r[2][12]), "=r"(r[2][13]), "=r"(r[2][14]), "=r"(r[2][15]), "=r"(r[2][16]), "=r"(r[2][17]), "=r"(r[2][18]), "=r"(r[2][19]), "=r"(r[2][20]), "=r"(r[2][21]), "=r"(r[2][22]), "=r"(r[2][23]), "=r"(r[2][24]), "=r"(r[2][25]), "=r"(r[2][26]), "=r"(r[2][27]), "=r"(r[2][28]), "=r"(r[2][29]), "=r"(r[2][30]), "=r"(r[2][31]), "=r"(r[3][0]), "=r"(r[3][1]), "=r"(r[3][2]), "=r"(r[3][3]), "=r"(r[3][4]), "=r"(r[3][5]), "=r"(r[3][6]), "=r"(r[3][7]), "=r"(r[3][8]), "=r"(r[3][9]), "=r"(r[3][10]), "=r"(r[3][11]), "=r"(r[3][12]), "=r"(r[3][13]), "=r"(r[3][14]), "=r"(r[3][15]), "=r"(r[3][16]), "=r"(r[3][17]), "=r"(r[3][18]), "=r"(r[3][19]), "=r"(r[3][20]), "=r"(r[3][21]), "=r"(r[3][22]), "=r"(r[3][23]), "=r"(r[3][24]), "=r"(r[3][25]), "=r"(r[3][26]), "=r"(r[3][27]), "=r"(r[3][28]), "=r"(r[3][29]), "=r"(r[3][30]), "=r"(r[3][31])
                 : "r"(taddr));
}
// As tmem_st32 for 64 consecutive columns in one instruction.
__device__ __forceinline__ void tmem_st64(uint32_t taddr, const uint32_t (&r)[2][32])
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64};\n" ::"r"(taddr), "r"(r[0][0]), "r"(r[0][1]), "r"(r[0][2]), "r"(r[0][3]), "r"(r[0][4]), "r"(r[0][5]), "r"(r[0][6]), "r"(r[0][7]), "r"(r[0][8]), "r"(r[0][9]), "r"(r[0][10]), "r"(r[0][11]), "r"(r[0][12]), "r"(r[0][13]), "r"(r[0][14]), "r"(r[0][15]), "r"(r[0][16]), "r"(r[0][17]), "r"(r[0][18]), "r"(r[0][19]), "r"(r[0][20]), "r"(r[0][21]), "r"(r[0][22]), "r"(r[0][23]), "r"(r[0][24]), "r"(r[0][25]), "r"(r[0][26]), "r"(r[0][27]), "r"(r[0][28]), "r"(r[0][29]), "r"(r[0][30]), "r"(r[0][31]), "r"(r[1][0]), "r"(r[1][1]), "r"(r[1][2]), "r"(r[1][3]), "r"(r[1][4]), "r"(r[1][5]), "r"(r[1][6]), "r"(r[1][7]), "r"(r[1][8]), "r"(r[1][9]), "r"(r[1][10]), "r"(r[1][11]), "r"(r[1][12]), "r"(r[1][13]), "r"(r[1][14]), "r"(r[1][15]), "r"(r[1][16]), "r"(r[1][17]), "r"(r[1][18]), "r"(r[1][19]), "r"(r[1][20]), "r"(r[1][21]), "r"(r[1][22]), "r"(r[1][23]), "r"(r[1][24]), "r"(r[1][25]), "r"(r[1][26]), "r"(r[1][27]), "r"(r[1][28]), "r"(r[1][29]), "r"(r[1][30]), "r"(r[1][31])
                 : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32])
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
                 "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
                 "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
                 "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
                 "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
                 "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
                 : "memory");
}
// 16 consecutive 32-bit columns of this thread's lane (warp-collective).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16])
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
                 "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
                 "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
                 : "memory");
}
// 16 columns of zeros (one zero register for every operand).
__device__ __forceinline__ void tmem_st16_zero(uint32_t taddr)
{
    const uint32_t z = 0u;
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
                 "{%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};\n" ::"r"(taddr), "r"(z)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
// Ties 32 registers to this point: code after it cannot read them earlier (placed after tmem_wait_ld, since the
// values of an asynchronous tcgen05.ld are only defined once the wait returns).
__device__ __forceinline__ void reg_fence(uint32_t (&r)[32])
{
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31]));
}
__device__ __forceinline__ void reg_fence16(uint32_t (&r)[16])
{
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]));
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

// Named barrier `id` (1 .. 15) over `count` threads (a multiple of 32).
__device__ __forceinline__ void named_bar(uint32_t id, uint32_t count)
{
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}
// Arrives at named barrier `id` without waiting (the producer side: shared-memory writes before it are seen by the
// threads that complete the barrier with named_bar).
__device__ __forceinline__ void named_arrive(uint32_t id, uint32_t count)
{
    asm volatile("bar.arrive %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}

// ---- packed fp32 arithmetic (sm_100) --------------------------------------------------------------------------------

__device__ __forceinline__ float max3f(float a, float b, float c)
{
    float d;
    asm("max.f32 %0, %1, %2, %3;\n" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
__device__ __forceinline__ uint64_t pack2(float lo, float hi)
{
    uint64_t d;
    asm("mov.b64 %0, {%1, %2};\n" : "=l"(d) : "f"(lo), "f"(hi));
    return d;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& lo, float& hi)
{
    asm("mov.b64 {%0, %1}, %2;\n" : "=f"(lo), "=f"(hi) : "l"(v));
}
// (a * b + c) on two fp32 lanes at once.
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c)
{
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;\n" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b)
{
    uint64_t d;
    asm("add.f32x2 %0, %1, %2;\n" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// ---- descriptors ---------------------------------------------------------------------------------------------------

// Shared-memory matrix descriptor (sm_100 UMMA): start address, leading / stride byte offsets, version 1, 128-byte
// swizzle.  Tiles are written by TMA with CU_TENSOR_MAP_SWIZZLE_128B from 1024-byte aligned bases.
//   K-major operand (rows of 64 16-bit values = 128 B): sbo = 1024 (8-row groups), lbo unused (16).
//   MN-major operand: lbo = bytes between 64-element blocks along M/N, sbo = 1024 (8-row groups along K).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo)
{
    uint64_t d = 0;
    d |= uint64_t((saddr & 0x3FFFF) >> 4);
    d |= uint64_t((lbo >> 4) & 0x3FFF) << 16;
    d |= uint64_t((sbo >> 4) & 0x3FFF) << 32;
    d |= uint64_t(1) << 46;  // descriptor version for sm_100
    d |= uint64_t(2) << 61;  // SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::f16 with fp32 accumulate: A / B element format (0 fp16, 1 bf16), major-ness
// (0 K-major, 1 MN-major), M and N.
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t a_fmt, uint32_t b_fmt, uint32_t a_mn, uint32_t b_mn,
                                                 uint32_t M, uint32_t N)
{
    return (1u << 4)            // D format fp32
           | (a_fmt << 7) | (b_fmt << 10) | (a_mn << 15) | (b_mn << 16) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// ---- tensor maps (host) -------------------------------------------------------------------------------------------

// cuTensorMapEncodeTiled, looked up once through the runtime (null where the driver does not provide it).
inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder()
{
    static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// [heads][rows][dim] 16-bit tiles as a TMA source: boxes of box_rows rows x 64 values (128 bytes, the 128-byte
// swizzle the UMMA descriptors above expect), zero fill past `rows`.
inline bool tile_map(CUtensorMap* map, const void* ptr, bool bf16, uint32_t dim, uint32_t rows, uint32_t heads,
                     uint32_t box_rows)
{
    auto enc = tensor_map_encoder();
    if (!enc)
        return false;
    cuuint64_t dims[3] = {dim, rows, heads};
    cuuint64_t strides[2] = {uint64_t(dim) * 2, uint64_t(rows) * dim * 2};
    cuuint32_t box[3] = {64, box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
               const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

} // namespace tc
} // namespace mako
