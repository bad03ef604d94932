// sm_100a building blocks for the attention kernels: mbarriers with bounded
// waits, TMA tile loads/stores, tcgen05 (UMMA) descriptors, MMA issue, commit,
// and TMEM allocation / load / store.  Everything here is inline PTX written
// for Blackwell datacenter parts (compute capability 10.0a); nothing falls back
// to older tensor-core paths.
//
// Shared-memory operand layout used throughout: every 16-bit tile of R rows by
// C columns (C a multiple of 64) is stored as C/64 consecutive "column blocks".
// A column block holds R rows of 128 bytes (64 elements) with the 128-byte
// swizzle: the 16-byte chunk index inside a row is XORed with (row % 8).  This
// is exactly what a TMA load with CU_TENSOR_MAP_SWIZZLE_128B and a box of
// {64, R} writes, and it is the canonical SWIZZLE_128B operand layout of
// tcgen05.mma in both K-major and MN-major form, so one tile can feed MMAs
// that read it either way (K-major as Q.K^T operand, MN-major as P.V operand).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace tk {

// Status codes shared by the kernels (device status word) and the C ABI.
enum : int {
  kOk = 0,
  kErrInvalidArgument = 1,
  kErrUnsupported = 2,
  kErrMisaligned = 3,
  kErrLaunch = 4,
  kErrTensorMap = 5,
  kErrDeviceTimeout = 6,
  kErrNoDriver = 7,
  kErrTooLarge = 8,
  kErrOutOfMemory = 9,
};

// Bytes of one swizzled column block row (64 16-bit elements).
constexpr int kSwizzleBytes = 128;
// Rows of every tile (query tile, key tile).
constexpr int kTileRows = 128;
// Bytes of one column block of a 128-row tile.
constexpr int kBlockBytes = kTileRows * kSwizzleBytes;  // 16 KiB

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t lane_id() {
  uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Per-CTA control block living in shared memory.  `abort` is raised by the
// first wait that runs out of time; every later wait in the CTA sees it and
// gives up at once, so a CTA whose pipeline broke drains in bounded time and
// still reaches its TMEM deallocation.
struct CtaControl {
  uint32_t tmem_base;
  volatile int abort;
};

// Wait for phase `parity` of `bar` to complete, for at most `timeout_ns`
// nanoseconds of wall time.  Returns false (after recording kErrDeviceTimeout
// in the global status word and raising the CTA abort flag) when the limit is
// reached or another warp of the CTA already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, CtaControl* ctl,
                                          uint64_t timeout_ns, int* status, int site) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t start = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(addr, parity)) return true;
    if (ctl->abort) return false;
    if ((++spins & 63u) == 0) {
      if (global_timer_ns() - start > timeout_ns) {
        ctl->abort = 1;
        if (status != nullptr) atomicCAS(status, kOk, kErrDeviceTimeout + (site << 8));
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor), no multicast anywhere.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0,
                                             int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_store_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void tma_store_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Wait until at most one committed bulk group still reads shared memory.
__device__ __forceinline__ void tma_store_wait_read_le1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

// Wait until every committed bulk group has fully completed (writes done).
__device__ __forceinline__ void tma_store_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Element-wise add of a shared-memory box into global memory (fp32 map),
// performed by the TMA unit; elements outside the tensor are skipped.
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, const void* src, int c0,
                                                  int c1, int c2) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], "
      "[%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Byte offset of fp32 element (row, col) inside one 128-byte-wide box
// (32 floats per row) stored with the 128-byte swizzle.
__device__ __forceinline__ uint32_t swz_offset_f32(uint32_t row, uint32_t col) {
  return row * kSwizzleBytes + ((((col >> 2) & 7u) ^ (row & 7u)) << 4) + ((col & 3u) << 2);
}

// Make this thread's generic-proxy shared-memory writes visible to the async
// proxy (TMA store, tcgen05.mma operand reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Programmatic dependent launch.  launch_dependents: this CTA no longer holds
// back the next kernel of the stream (launched with programmatic stream
// serialization), which may start its prologue; wait_prerequisites: block
// until every grid this one depends on has completed and its memory writes
// are visible.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_prerequisites() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Byte offset of element (row, col) of a 16-bit tile in the swizzled
// column-block layout described at the top of this file.
__device__ __forceinline__ uint32_t swz_offset(uint32_t row, uint32_t col, uint32_t rows) {
  const uint32_t block = col >> 6;
  const uint32_t chunk = (col >> 3) & 7u;
  return block * rows * kSwizzleBytes + row * kSwizzleBytes + ((chunk ^ (row & 7u)) << 4) +
         ((col & 7u) << 1);
}

// ---------------------------------------------------------------------------
// tcgen05: descriptors
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor (sm_100 format): start address, leading and
// stride byte offsets (all >> 4), descriptor version 1 at bit 46, layout
// SWIZZLE_128B (2) in bits 61..63.  base_offset stays 0 because every tile
// starts on a 1024-byte boundary.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// K-major operand: rows are M (or N), the 16-bit K elements of a row are
// contiguous.  k is the first K element of this MMA (multiple of 16).
__device__ __forceinline__ uint64_t sdesc_kmajor(uint32_t tile_saddr, uint32_t rows, uint32_t k) {
  const uint32_t addr = tile_saddr + (k >> 6) * rows * kSwizzleBytes + (k & 63u) * 2u;
  return sdesc_sw128(addr, 16u, 8u * kSwizzleBytes);
}

// MN-major operand: the tile rows are K, the 16-bit M (or N) elements of a row
// are contiguous (64 per column block).  k is the first K row of this MMA.
__device__ __forceinline__ uint64_t sdesc_mnmajor(uint32_t tile_saddr, uint32_t rows, uint32_t k) {
  const uint32_t addr = tile_saddr + k * kSwizzleBytes;
  return sdesc_sw128(addr, rows * kSwizzleBytes, 8u * kSwizzleBytes);
}

// Instruction descriptor for kind::f16 with an f32 accumulator.
// fmt: 0 = f16, 1 = bf16 (A and B always share one type).
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t fmt, uint32_t m, uint32_t n,
                                                 uint32_t a_mn_major, uint32_t b_mn_major) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (a_mn_major << 15) | (b_mn_major << 16) |
         ((n >> 3) << 17) | ((m >> 4) << 24);
}

// ---------------------------------------------------------------------------
// tcgen05: MMA issue / commit / fences
// ---------------------------------------------------------------------------
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// A operand read from TMEM (M lanes x K/2 columns of packed 16-bit pairs).
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same SW128 descriptors split into two 32-bit words.  The high word
// (stride byte offset 1024, version 1, SWIZZLE_128B) is the same for every
// operand here; the low word holds the start address (>> 4) and the leading
// byte offset.  Within a tile only the start address changes from one MMA
// to the next, and shared addresses stay below 256 KB, so a per-MMA low word
// is `base + constant` with no carry into the offset field: the issuing
// thread spends one add per operand per MMA.
constexpr uint32_t kSdescHi = (1024u >> 4) | (1u << 14) | (2u << 29);
__device__ __forceinline__ uint32_t sdesc_lo_kmajor(uint32_t tile_saddr) {
  return ((tile_saddr >> 4) & 0x3FFFu) | ((16u >> 4) << 16);
}
__device__ __forceinline__ uint32_t sdesc_lo_mnmajor(uint32_t tile_saddr, uint32_t rows) {
  return ((tile_saddr >> 4) & 0x3FFFu) | (((rows * kSwizzleBytes) >> 4) << 16);
}
// Start-address increments (16-byte units) of K element k (a multiple of 16).
__host__ __device__ constexpr uint32_t kmajor_koff(uint32_t rows, uint32_t k) {
  return ((k >> 6) * rows * kSwizzleBytes + (k & 63u) * 2u) >> 4;
}
__host__ __device__ constexpr uint32_t mnmajor_koff(uint32_t k) { return (k * kSwizzleBytes) >> 4; }

__device__ __forceinline__ void umma_ss_w(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "mov.b64 da, {%1, %5};\n\t"
      "mov.b64 db, {%2, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_lo), "r"(b_lo), "r"(idesc), "r"(accumulate), "r"(kSdescHi)
      : "memory");
}

__device__ __forceinline__ void umma_ts_w(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 db;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "mov.b64 db, {%2, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "r"(b_lo), "r"(idesc), "r"(accumulate), "r"(kSdescHi)
      : "memory");
}

// One lane of a converged warp (elect.sync): the lane that issues
// single-thread tcgen05 operations while the whole warp runs the loop.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// Arrive once on `bar` when every tcgen05.mma previously issued by this
// thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation (whole warp) and data movement (whole warp)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(dst_smem)),
      "r"(ncols)
      : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t receives lane (base+t).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void reg_fence16(uint32_t (&r)[16]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]),
                 "+r"(r[13]), "+r"(r[14]), "+r"(r[15]));
}

// Ties 32 registers written by tcgen05.ld to a point after tcgen05.wait::ld:
// the compiler cannot move any use of them above this (empty) statement.
__device__ __forceinline__ void reg_fence(uint32_t (&r)[32]) {
  asm volatile("" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

// ---------------------------------------------------------------------------
// Per-warpgroup register reallocation.  Every warp of the warpgroup executes
// it.  `inc` blocks until the registers released by `dec` elsewhere in the CTA
// are available, so the shares must add up to the launch allocation
// (threads x registers per thread); launchers check that allocation first.
// ---------------------------------------------------------------------------
template <int kRegs>
__device__ __forceinline__ void warpgroup_reg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegs));
}
template <int kRegs>
__device__ __forceinline__ void warpgroup_reg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegs));
}

// ---------------------------------------------------------------------------
// Numerics helpers
// ---------------------------------------------------------------------------
// Hardware base-2 exponential (MUFU.EX2), flushes denormals; exp2(-inf) = +0.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---------------------------------------------------------------------------
// Packed fp32 pairs (sm_100 fma/add/mul .f32x2: two lanes of fp32 work per
// issued instruction).  A pair lives in a 64-bit register, `lo` first.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Two base-2 exponentials on the FMA pipe with packed arithmetic (about five
// issued instructions per exponential), for splitting a softmax's
// exponentials between the MUFU (16 per clock per SM) and the FP32 units.
// Method (Cody-Waite style range reduction): n = round(x) from the low
// mantissa bits of x + 1.5*2^23, f = x - n in [-1/2, 1/2], n added to the
// exponent field of 2^f, which comes from a degree-3
// polynomial for 2^f fitted here for minimum relative error on [-1/2, 1/2]
// (Lawson-weighted least squares; max relative error 7.5e-5 in fp32 Horner
// form, below the 2^-11 rounding of the 16-bit P it feeds) wherever the
// result is a normal float (x in [-125.5, 127]); in [-126, -125.5) a result
// just below 2^-126 comes out subnormal, relative error up to 1.5e-4.
// Inputs below -126 are clamped (result in [0, 2^-126] instead of 0); valid
// for x <= 127.  tests/test_exp2_fma.py checks these bounds.
__device__ __forceinline__ void exp2_fma_pair(float x0, float x1, float& p0, float& p1) {
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
  const uint64_t x = f2_pack(fmaxf(x0, -126.0f), fmaxf(x1, -126.0f));
  const uint64_t t = fadd2(x, f2_pack(kShift, kShift));
  const uint64_t n = fadd2(t, f2_pack(-kShift, -kShift));
  const uint64_t f = ffma2(n, f2_pack(-1.0f, -1.0f), x);
  uint64_t p = ffma2(f, f2_pack(5.517132208e-02f, 5.517132208e-02f), f2_pack(2.426105440e-01f, 2.426105440e-01f));
  p = ffma2(p, f, f2_pack(6.932609677e-01f, 6.932609677e-01f));
  p = ffma2(p, f, f2_pack(9.999281168e-01f, 9.999281168e-01f));
  float q0, q1, t0, t1;
  f2_unpack(p, q0, q1);
  f2_unpack(t, t0, t1);
  p0 = __uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23));
  p1 = __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23));
}

// 32-byte global store of eight 32-bit words (sm_100 st.global.v8); `dst`
// must be 32-byte aligned.
__device__ __forceinline__ void st_global_v8(void* dst, const uint32_t* w) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst), "r"(w[0]), "r"(w[1]),
               "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}

// Three-input maximum (sm_100 max.f32 with three sources).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Pack two floats into one 32-bit word of 16-bit values, `lo` in bits 0..15
// (the even K element of a tcgen05 A operand pair).
template <bool kBf16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (kBf16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

}  // namespace tk
