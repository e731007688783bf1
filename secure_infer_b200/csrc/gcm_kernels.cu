// gcm_kernels.cu -- sm_100a kernels of the authenticated KV transfer path.
//
//   gcm_schedule_kernel      per-key AES round keys + the GHASH nibble tables
//   gcm_layer_ctr_kernel     keystream + tag masks of a layer's records
//   gcm_layer_verify_kernel  warp-segmented GHASH fused with CTR XOR, the
//                            fail-closed gate, int8/int4 -> bf16 dequantisation
//                            and the block-table scatter; in encrypt mode the
//                            writeback mirror (XOR, GHASH, tag, record layout)
//   kv_encode_kernel         writeback quantisation of bf16 KV blocks into packets
//   gcm_segment_kernel       plugin ABI: CTA-segmented GCM over up to four
//                            descriptor records (decrypt/verify/encrypt/GHASH/XOR)
//   gcm_ctr_kernel           plugin ABI: AES-CTR keystream or CTR XOR jobs
//   auth_gate_kernel         zero a buffer whose status is not 1
//
// Semantics follow the reference AICPU kernels
// (secure_infer/native/kernels/aicpu/ghash.aicpu): counter blocks :133-147,
// decrypt_verify :594-651, encrypt_tag :656-699, verify_xor :705-773,
// verify_only :780-827, verify_xor_batch :834-940, xor_only :948-976,
// ghash :978-1046, auth_gate :1051-1068; and the reference codec
// (secure_infer/kv_offload/transport_codec.py:22-42, optimized_decode.py:5-27).
#include "gcm_device.cuh"
#include "gcm_kernels.cuh"
#include "bitsliced_aes.cuh"
#include "kx.cuh"

#include <cuda_bf16.h>

#include <atomic>
#include <cstddef>
#include <mutex>
#include <vector>

namespace sib {

// ----------------------------------------------------------------------------
// Warp helpers
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint4 shfl_xor4(uint4 v, int m)
{
    return make_uint4(__shfl_xor_sync(0xffffffffu, v.x, m), __shfl_xor_sync(0xffffffffu, v.y, m),
                      __shfl_xor_sync(0xffffffffu, v.z, m), __shfl_xor_sync(0xffffffffu, v.w, m));
}

// Quarter stage of the segment combine: every lane of an active quarter holds
// the quarter sum V, and the quarter returns V * M (M's nibble table tab,
// entry p * 16 + v) in all its lanes.  Lane r of the quarter looks up nibbles
// 4 r .. 4 r + 3 and the quarter XOR-reduces: 4 LDS.128 per lane instead of 32
// for a lane-by-lane product.  Every lane must call it (the reduction
// shuffles); lanes of an inactive quarter return zero.
__device__ __forceinline__ uint4 gf_mul_quarter(uint4 v, const uint4* __restrict__ tab, uint32_t rep, bool active)
{
    const uint32_t wi = rep >> 1;
    const uint32_t w = wi == 0 ? v.x : wi == 1 ? v.y : wi == 2 ? v.z : v.w;
    const uint32_t half = (rep & 1u) * 16u;
    uint4 acc = zero4();
    if (active) {
#pragma unroll
        for (uint32_t i = 0; i < 4; ++i) {
            // nibble p = 4 r + i: byte 2 r + i / 2, high nibble for even p.
            const uint32_t shift = half + (i >> 1) * 8u + ((i & 1u) ? 0u : 4u);
            acc = xor4(acc, tab[(4u * rep + i) * 16u + ((w >> shift) & 0xfu)]);
        }
    }
    acc = xor4(acc, shfl_xor4(acc, 1));
    acc = xor4(acc, shfl_xor4(acc, 2));
    return xor4(acc, shfl_xor4(acc, 4));
}

__device__ __forceinline__ uint4 shfl_up4(uint4 v, uint32_t d)
{
    return make_uint4(__shfl_up_sync(0xffffffffu, v.x, d), __shfl_up_sync(0xffffffffu, v.y, d),
                      __shfl_up_sync(0xffffffffu, v.z, d), __shfl_up_sync(0xffffffffu, v.w, d));
}

__device__ __forceinline__ uint4 warp_xor_reduce(uint4 v)
{
#pragma unroll
    for (int m = 16; m; m >>= 1) v = xor4(v, shfl_xor4(v, m));
    return v;
}

// z * M with the 32 lanes of a warp each doing one nibble lookup; z must be
// warp-uniform.  tab is an unreplicated table (shared or global).
template <bool kGlobal>
__device__ __forceinline__ uint4 gf_mul_warp(uint4 z, const uint4* tab, int lane)
{
    const uint4* p = tab + lane * 16 + nibble_le(z, lane);
    return warp_xor_reduce(kGlobal ? __ldg(p) : *p);
}

__device__ __forceinline__ uint4 len_block_le(uint32_t aad_bytes, uint64_t count)
{
    const uint64_t a = static_cast<uint64_t>(aad_bytes) * 8u, c = count * 8u;
    return make_uint4(bswap32(static_cast<uint32_t>(a >> 32)), bswap32(static_cast<uint32_t>(a)),
                      bswap32(static_cast<uint32_t>(c >> 32)), bswap32(static_cast<uint32_t>(c)));
}

__device__ __forceinline__ uint4 j0_block_le(const uint32_t iv[4])
{
    return make_uint4(bswap32(iv[0]), bswap32(iv[1]), bswap32(iv[2]), bswap32(1u));
}

__device__ __forceinline__ uint4 mask_bytes(uint4 v, uint64_t avail)
{
    if (avail >= 16) return v;
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
    for (int i = 0; i < 4; ++i) {
        const int64_t keep = static_cast<int64_t>(avail) - 4 * i;
        const uint32_t m = keep >= 4 ? 0xffffffffu : keep <= 0 ? 0u : ((1u << (8 * keep)) - 1u);
        w[i] &= m;
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ void store_block(uint8_t* p, uint4 v, uint64_t avail, bool aligned)
{
    if (aligned && avail >= 16) *reinterpret_cast<uint4*>(p) = v;
    else store_partial16(p, v, avail);
}

__device__ __forceinline__ bool equal4(uint4 a, uint4 b) { return is_zero4(xor4(a, b)); }

// 16-byte global -> shared asynchronous copy (bypasses registers and L1).
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src)
{
    const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(gmem_src) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all()
{
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// Wait until at most N of this thread's committed copy groups are pending.
template <int N>
__device__ __forceinline__ void cp_async_wait_group()
{
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// mbarrier + bulk (TMA, non-multicast) global -> shared copy of this GPU's
// own memory.  Used to fetch tables in the background of a kernel's main loop.
__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init_expect(uint64_t* bar, uint32_t tx_bytes)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n"
                 "fence.mbarrier_init.release.cluster;\n"
                 "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(tx_bytes)
                 : "memory");
}

// Bulk prefetch of [p, p + bytes) into L2 (16-byte aligned, bytes a multiple of
// 16): no completion to wait for, no registers or shared memory held.
__device__ __forceinline__ void l2_prefetch_bulk(const void* p, uint32_t bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(smem_dst)),
                 "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Waits for phase `parity` of the barrier; gives up after a bounded number of
// polls (returns false) so a lost completion can never hang the GPU.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity)
{
    for (uint32_t it = 0; it < (1u << 22); ++it) {
        uint32_t done;
        asm volatile("{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}"
                     : "=r"(done)
                     : "r"(smem_u32(bar)), "r"(parity)
                     : "memory");
        if (done) return true;
    }
    return false;
}

// ----------------------------------------------------------------------------
// Key schedule: one CTA of 8 warps.  Reuses the previous build when the key
// (and H) bytes are unchanged, so per-call plugin launches stay cheap.
// ----------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gcm_schedule_kernel(const uint8_t* key, const uint8_t* h,
                                                           GcmSchedule* S, int need_tables)
{
    __shared__ uint4 tab_s[32 * 16];
    __shared__ uint4 pow_le[kGhashTables];
    __shared__ uint4 pow_hi[5];               // H^(2^13) .. H^(2^17)
    __shared__ int s_skip;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    if (tid == 0) {
        bool same = S->valid == 1u;
        if (key) {
            same = same && S->reserved[1] == 1u;
            for (int i = 0; i < 16; ++i) same = same && S->key_copy[i] == key[i];
        }
        if (need_tables) {
            same = same && S->reserved[0] == 1u && S->h_from_key == (h == nullptr ? 1u : 0u);
            if (h) for (int i = 0; i < 16; ++i) same = same && S->h_copy[i] == h[i];
        }
        s_skip = same ? 1 : 0;
    }
    __syncthreads();
    if (s_skip) return;

    if (tid == 0) {
        uint32_t rk[44] = {};
        if (key) {
            aes128_expand_le(key, rk);
            for (int i = 0; i < 16; ++i) S->key_copy[i] = key[i];
        }
        S->reserved[1] = key ? 1u : 0u;   // round keys valid
        for (int i = 0; i < 44; ++i) S->rk[i] = rk[i];
        uint4 hv = zero4();
        if (h) {
            hv = load_partial16(h, 16);
            for (int i = 0; i < 16; ++i) S->h_copy[i] = h[i];
        } else {
            hv = aes128_encrypt_global(zero4(), rk);   // H = E_K(0^128)
        }
        S->h_le = hv;
        S->h_from_key = h == nullptr ? 1u : 0u;
        S->reserved[0] = 0u;
        pow_le[0] = hv;
    }
    __syncthreads();
    if (!need_tables) {
        if (tid == 0) { __threadfence(); S->valid = 1u; }
        return;
    }
    if (warp == 0) {
        // H^2..H^32 by repeated multiplication with H's table.
        build_nibble_table_warp(bswap4(pow_le[0]), tab_s, lane);
        __syncwarp();
        uint4 cur = pow_le[0];
        for (int e = 2; e <= 32; ++e) {
            cur = gf_mul_warp<false>(cur, tab_s, lane);
            if (lane == 0) pow_le[tab_pow_small(e)] = cur;
        }
        __syncwarp();
        // H^64..H^2048 with H^32's table.
        build_nibble_table_warp(bswap4(cur), tab_s, lane);
        __syncwarp();
        for (int k = 2; k <= 64; ++k) {
            cur = gf_mul_warp<false>(cur, tab_s, lane);
            if (lane == 0) pow_le[tab_pow_32k(k)] = cur;
        }
        // H^4096 = (H^2048)^2.
        __syncwarp();
        build_nibble_table_warp(bswap4(cur), tab_s, lane);
        __syncwarp();
        cur = gf_mul_warp<false>(cur, tab_s, lane);
        if (lane == 0) pow_le[kTabSeg] = cur;
        // H^(2^13) .. H^(2^17) by squaring, for the plugin kernel's segment joins.
        for (int e = 0; e < 5; ++e) {
            __syncwarp();
            build_nibble_table_warp(bswap4(cur), tab_s, lane);
            __syncwarp();
            cur = gf_mul_warp<false>(cur, tab_s, lane);
            if (lane == 0) pow_hi[e] = cur;
        }
    }
    __syncthreads();
    for (int t = warp; t < kGhashTables; t += 8) build_nibble_table_warp(bswap4(pow_le[t]), S->tab[t], lane);
    if (warp < 5) build_nibble_table_warp(bswap4(pow_hi[warp]), S->pow2hi[warp], lane);
    __syncthreads();
    // Shared-memory-ready layouts for the layer kernel.
    for (int i = tid; i < 32 * 16 * 8; i += 256) {
        const int e = i >> 3, r = i & 7;
        S->lane8[i] = S->tab[tab_pow_small(8 - r)][e];
        // byte32 entry i: position b = (i >> 11) * 8 + (i & 7), value v = (i >> 3) & 255;
        // byte b holds nibbles 2b (high) and 2b + 1 (low).
        const int b = (i >> 11) * 8 + (i & 7), v = (i >> 3) & 255;
        const uint4* t32 = S->tab[tab_pow_small(32)];
        S->byte32[i] = xor4(t32[(2 * b) * 16 + (v >> 4)], t32[(2 * b + 1) * 16 + (v & 15)]);
        const uint4* t256 = S->tab[kTabStride];
        S->byte256[i] = xor4(t256[(2 * b) * 16 + (v >> 4)], t256[(2 * b + 1) * 16 + (v & 15)]);
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        S->reserved[0] = 1u;
        S->valid = 1u;
    }
}

// Segment join tables for the layer kernels: for every segment length
// L = 32 s blocks (s = 1..kMaxWarpSegSteps), the nibble tables of
// H^(L 2^b), b = 1..5, at out[((s - 1) * 5 + b - 1) * 512].  One warp per s,
// by repeated squaring from H^(32 s).  Built once per session key.
__global__ void __launch_bounds__(32) gcm_join_tables_kernel(const GcmSchedule* S, uint4* out)
{
    const int s = blockIdx.x + 1, lane = threadIdx.x;
    const uint4* tab = S->tab[tab_pow_32k(s)];
    uint4 v = tab[8];                 // entry (0, 8) = the multiplier itself, LE layout
    for (int b = 1; b <= 5; ++b) {
        v = gf_mul_warp<false>(v, tab, lane);
        uint4* dst = out + ((s - 1) * 5 + b - 1) * 512;
        build_nibble_table_warp(bswap4(v), dst, lane);
        __syncwarp();
        tab = dst;
    }
}

// ----------------------------------------------------------------------------
// AES-CTR keystream / payload XOR.
// ----------------------------------------------------------------------------
__device__ __forceinline__ void fill_aes_smem(uint32_t* te, uint32_t* rk, const GcmSchedule* S)
{
    uint4* te4 = reinterpret_cast<uint4*>(te);
    for (uint32_t i = threadIdx.x; i < 2048; i += blockDim.x) {
        const uint32_t t = kAesDev.te0[i >> 3];
        te4[i] = make_uint4(t, t, t, t);
    }
    if (threadIdx.x < 44) rk[threadIdx.x] = S->rk[threadIdx.x];
}

// Four replicated T-tables (Te_t = rotl(te0, 8t)) laid out so that one PRMT
// forms a lookup's shared-memory address: byte 0 = lane * 4 (+128 for odd t),
// byte 1 = the state byte v, byte 2 = t >> 1.  Table pair (Te0, Te1) fills
// [0, 64 KiB), pair (Te2, Te3) fills [64 KiB, 128 KiB); every lane reads its
// own bank, so a warp's 32 lookups are one conflict-free wavefront.
constexpr uint32_t kCtrThreads = 1024;
// The layer keystream kernel uses half the register file (512 threads x 64),
// so a quantise CTA of the writeback path can share the SM with it.
constexpr uint32_t kLayerCtrThreads = 512;
constexpr size_t kCtrTableBytes = 131072;
constexpr size_t kCtrSmem = kCtrTableBytes + 256;

struct Aes4Tables {
    const uint8_t* smem;
    uint32_t base[4];
    __device__ __forceinline__ uint32_t look(int t, uint32_t s, int k) const
    {
        const uint32_t addr = __byte_perm(s, base[t], 0x7604u | (static_cast<uint32_t>(k) << 4));
        return *reinterpret_cast<const uint32_t*>(smem + addr);
    }
};

// Rounds first .. 10 of AES-128 on state s (the output of round first - 1).
__device__ __forceinline__ uint4 aes128_rounds_from(uint4 s, int first, const Aes4Tables& T,
                                                    const uint32_t* __restrict__ rk)
{
    uint32_t s0 = s.x, s1 = s.y, s2 = s.z, s3 = s.w;
#pragma unroll
    for (int r = first; r < 10; ++r) {
        const uint4 k4 = make_uint4(rk[4 * r], rk[4 * r + 1], rk[4 * r + 2], rk[4 * r + 3]);
        const uint32_t t0 = T.look(0, s0, 0) ^ T.look(1, s1, 1) ^ T.look(2, s2, 2) ^ T.look(3, s3, 3) ^ k4.x;
        const uint32_t t1 = T.look(0, s1, 0) ^ T.look(1, s2, 1) ^ T.look(2, s3, 2) ^ T.look(3, s0, 3) ^ k4.y;
        const uint32_t t2 = T.look(0, s2, 0) ^ T.look(1, s3, 1) ^ T.look(2, s0, 2) ^ T.look(3, s1, 3) ^ k4.z;
        const uint32_t t3 = T.look(0, s3, 0) ^ T.look(1, s0, 1) ^ T.look(2, s1, 2) ^ T.look(3, s2, 3) ^ k4.w;
        s0 = t0; s1 = t1; s2 = t2; s3 = t3;
    }
    // Final round: S(x) sits in byte 0 of Te2, byte 1 of Te3, byte 2 of Te0,
    // byte 3 of Te1; PRMT gathers the four bytes of each output column.
    const uint4 k4 = make_uint4(rk[40], rk[41], rk[42], rk[43]);
    auto column = [&](uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
        const uint32_t lo = __byte_perm(T.look(2, a, 0), T.look(3, b, 1), 0x0050u);
        const uint32_t hi = __byte_perm(T.look(0, c, 2), T.look(1, d, 3), 0x7200u);
        return __byte_perm(lo, hi, 0x7610u);
    };
    return make_uint4(column(s0, s1, s2, s3) ^ k4.x, column(s1, s2, s3, s0) ^ k4.y,
                      column(s2, s3, s0, s1) ^ k4.z, column(s3, s0, s1, s2) ^ k4.w);
}

__device__ __forceinline__ uint4 aes128_encrypt_t4(uint4 in, const Aes4Tables& T, const uint32_t* __restrict__ rk)
{
    return aes128_rounds_from(make_uint4(in.x ^ rk[0], in.y ^ rk[1], in.z ^ rk[2], in.w ^ rk[3]), 1, T, rk);
}

// The same AES as a call, for rare blocks (general-path steps, tag masks), so
// a kernel carries one copy of it besides its unrolled main loop.
__device__ __noinline__ uint4 aes128_encrypt_t4_call(uint4 in, const Aes4Tables T, const uint32_t* rk)
{
    return aes128_encrypt_t4(in, T, rk);
}

__device__ __forceinline__ void fill_aes4_smem(uint8_t* smem, const GcmSchedule* S)
{
    uint4* s4 = reinterpret_cast<uint4*>(smem);
    for (uint32_t i = threadIdx.x; i < kCtrTableBytes / 16; i += blockDim.x) {
        const uint32_t off = i * 16u;
        const uint32_t v = (off >> 8) & 0xffu;
        const uint32_t t = ((off >> 16) << 1) | ((off >> 7) & 1u);
        const uint32_t val = rotl32(kAesDev.te0[v], static_cast<int>(8 * t));
        s4[i] = make_uint4(val, val, val, val);
    }
    uint32_t* rk = reinterpret_cast<uint32_t*>(smem + kCtrTableBytes);
    if (threadIdx.x < 44) rk[threadIdx.x] = S->rk[threadIdx.x];
}

__device__ __forceinline__ Aes4Tables aes4_view(const uint8_t* smem)
{
    const uint32_t lane4 = (threadIdx.x & 31u) * 4u;
    return Aes4Tables{smem, {lane4, lane4 | 128u, 0x10000u | lane4, 0x10000u | lane4 | 128u}};
}

__global__ void __launch_bounds__(kCtrThreads, 1) gcm_ctr_kernel(const __grid_constant__ CtrLaunch L,
                                                                  uint64_t uniform_blocks)
{
    extern __shared__ __align__(16) uint8_t smem[];
    fill_aes4_smem(smem, L.sched);
    __syncthreads();
    const uint32_t* rk = reinterpret_cast<const uint32_t*>(smem + kCtrTableBytes);
    const Aes4Tables T = aes4_view(smem);
    const CtrJob* jobs = L.jobs ? L.jobs : L.inl;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t gb = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; gb < L.total_blocks;
         gb += stride) {
        uint32_t j;
        if (uniform_blocks) {
            j = static_cast<uint32_t>(gb / uniform_blocks);
        } else {
            uint32_t lo = 0, hi = L.njobs - 1;
            while (lo < hi) {
                const uint32_t mid = (lo + hi + 1) >> 1;
                if (jobs[mid].block_first <= gb) lo = mid; else hi = mid - 1;
            }
            j = lo;
        }
        const CtrJob& J = jobs[j];
        const uint64_t c = gb - J.block_first;
        const uint64_t off = c * 16u;
        const uint64_t avail = J.bytes - off;
        uint4 ks = aes128_encrypt_t4(ctr_block_le(J.iv, c), T, rk);
        const bool aligned = !L.unaligned;
        if (J.in) ks = xor4(ks, (aligned && avail >= 16) ? ldg16(J.in + off) : load_partial16(J.in + off, avail));
        store_block(J.out + off, ks, avail, aligned);
    }
}

// ----------------------------------------------------------------------------
// Segmented GCM kernel.
// ----------------------------------------------------------------------------
// Work item = (record, segment).  The block sequence X = AAD || payload || len
// (m blocks) is cut into segments aligned to its END: the last nseg-1 segments
// hold SB blocks (256..4096, chosen per launch so small calls still spread over
// the SMs), the first holds the remaining len0 blocks.  Thread t
// of the CTA takes blocks base + t + 256 j (coalesced) and runs Horner with
// H^256; the 256 partials are scaled to S_seg = sum_t Y_t H^(256-t) (see the
// schedule comment).  Leading zero blocks (base < segment start) leave a
// zero-started GHASH unchanged.  The last CTA of a record to finish joins the
// segment partials with H^SB (staged in shared memory), derives E_K(J0),
// checks/emits the tag
// and, on authentication failure, zeroes everything the record wrote
// ("write then gate": nothing is released before the stream reaches the
// layer event recorded after this kernel).
constexpr int kBatch = 8;
constexpr size_t kGhashSmem = 4096 * sizeof(uint4);          // H^256 (plugin) or H^32 (layer) byte tables
constexpr size_t kAesSmem = 256 * 32 * sizeof(uint32_t) + 256; // T-table replicas + round keys
template <bool kInlineAes>
__global__ void __launch_bounds__(kThreads, 2) gcm_segment_kernel(const __grid_constant__ SegmentLaunch L)
{
    extern __shared__ __align__(16) uint8_t smem[];
    uint4* gtab = reinterpret_cast<uint4*>(smem);
    uint32_t* aes_te = reinterpret_cast<uint32_t*>(smem + kGhashSmem);
    uint32_t* aes_rk = aes_te + 256 * 32;
    __shared__ uint4 red[kThreads];
    __shared__ uint32_t s_last, s_ok;

    const GcmSchedule* __restrict__ S = L.sched;
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5, rep = lane & 7u;
    // The Horner multiplier H^256 as byte tables (64 KiB) by one bulk copy,
    // overlapping the AES table fill; waited for (bounded) before the first
    // GHASH step.  A copy that never lands poisons the partials, so records
    // fail closed.
    __shared__ __align__(8) uint64_t gtab_bar;
    if (tid == 0) {
        mbar_init_expect(&gtab_bar, 65536u);
        bulk_g2s(gtab, S->byte256, 65536u, &gtab_bar);
    }
    if constexpr (kInlineAes) fill_aes_smem(aes_te, aes_rk, S);
    __syncthreads();
    const bool gtab_ready = mbar_wait_bounded(&gtab_bar, 0);
    const GcmRecord* recs = L.recs ? L.recs : L.inl;
    const SmemAes aes{aes_te, aes_rk, lane};
    // Segment length SB (256..4096 blocks) and its join table H^SB.
    const int64_t SB = L.seg_blocks ? L.seg_blocks : kSegBlocks;

    for (uint32_t w = blockIdx.x; w < L.total_segs; w += gridDim.x) {
        uint32_t lo = 0, hi = L.nrec - 1;
        while (lo < hi) {
            const uint32_t mid = (lo + hi + 1) >> 1;
            if (recs[mid].seg_first <= w) lo = mid; else hi = mid - 1;
        }
        const uint32_t r = lo;
        const GcmRecord& R = recs[r];
        const uint32_t op = R.op, flags = R.flags, nseg = R.nseg;
        const uint64_t count = R.count;
        const uint32_t aad_bytes = R.aad_bytes;
        const uint8_t* in = R.in;
        const uint8_t* ksp = R.ks;
        uint8_t* out = R.out;
        const bool aligned = (flags & kRecUnaligned) == 0;

        const int64_t a_blk = (aad_bytes + 15) >> 4;
        const int64_t n_blk = static_cast<int64_t>((count + 15) >> 4);
        const int64_t m = a_blk + n_blk + 1;
        const uint32_t k = w - R.seg_first;
        const int64_t len0 = m - static_cast<int64_t>(nseg - 1) * SB;
        const int64_t seg_end = len0 + static_cast<int64_t>(k) * SB;
        const int64_t seg_len = k == 0 ? len0 : SB;
        const int J = static_cast<int>((seg_len + kThreads - 1) / kThreads);
        const int64_t base = seg_end - static_cast<int64_t>(J) * kThreads;

        uint4 Y = zero4();
        for (int jb = 0; jb < J; jb += kBatch) {
            uint4 xin[kBatch], kin[kBatch];
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
                xin[u] = zero4();
                kin[u] = zero4();
                const int j = jb + u;
                const int64_t i = base + tid + static_cast<int64_t>(j) * kThreads;
                if (j >= J || i < 0) continue;
                if (i < a_blk) {
                    xin[u] = load_partial16(R.aad + 16 * i, aad_bytes - 16 * i);
                } else if (i < a_blk + n_blk) {
                    const uint64_t off = static_cast<uint64_t>(i - a_blk) * 16u;
                    const uint64_t avail = count - off;
                    if (aligned && avail >= 16) {
                        xin[u] = ldg16(in + off);
                        if (ksp) kin[u] = ldg16(ksp + off);
                    } else {
                        xin[u] = load_partial16(in + off, avail);
                        if (ksp) kin[u] = load_partial16(ksp + off, avail);
                    }
                } else {
                    xin[u] = len_block_le(aad_bytes, count);
                }
            }
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
                const int j = jb + u;
                if (j >= J) break;
                const int64_t i = base + tid + static_cast<int64_t>(j) * kThreads;
                uint4 X = xin[u];
                if (i >= a_blk && i < a_blk + n_blk) {
                    const uint64_t c = static_cast<uint64_t>(i - a_blk);
                    const uint64_t off = c * 16u;
                    const uint64_t avail = count - off;
                    uint4 ks = kin[u];
                    if constexpr (kInlineAes) {
                        if (!ksp) ks = aes.encrypt(ctr_block_le(R.iv, c));
                    }
                    if (op == kOpDecrypt) {
                        store_block(out + off, xor4(X, ks), avail, aligned);
                    } else if (op == kOpEncrypt) {
                        const uint4 C = mask_bytes(xor4(X, ks), avail);
                        store_block(out + off, C, avail, aligned);
                        X = C;
                    } else if (op == kOpXorOnly || (op == kOpGhash && (flags & kGhashXorOnSuccess))) {
                        store_block(out + off, xor4(X, ks), avail, aligned);
                    }
                }
                if (op != kOpXorOnly) Y = j == 0 ? X : xor4(gf_mul_byte8(Y, gtab, rep), X);
            }
        }

        if (op != kOpXorOnly) {
            if (!gtab_ready) Y = make_uint4(~0u, ~0u, ~0u, ~0u);
            if (warp != 7) Y = gf_mul_table<1, true>(Y, S->tab[tab_pow_32k(7 - warp)], 0);
            red[tid] = Y;
            __syncthreads();
            if (warp == 0) {
                uint4 U = red[lane];
#pragma unroll
                for (int ww = 1; ww < 8; ++ww) U = xor4(U, red[ww * 32 + lane]);
                U = gf_mul_table<1, true>(U, S->tab[tab_pow_small(32 - lane)], 0);
                U = warp_xor_reduce(U);
                if (lane == 0) L.partials[w] = U;
            }
        }
        // Publish this segment: every thread's output stores, then the partial.
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const uint32_t prev = atomicAdd(&L.counters[r], 1u);
            s_last = prev == nseg - 1 ? 1u : 0u;
        }
        __syncthreads();
        if (!s_last) continue;

        __threadfence();
        // Join the record's partials, S = sum_k p_k H^(SB (nseg - 1 - k)).  SB
        // is a power of two 2^e0, so every power needed is some H^(2^e).  The
        // five tables H^(SB 2^b), b = 0..4, go into the Horner table's shared
        // memory (this CTA's main loop is done); chunks of 32 partials (the
        // first takes the remainder) are reduced by a lane tree, up to eight
        // chunks at a time on the eight warps, and warp 0 joins the chunk
        // values with H^(32 SB).
        uint4 acc = zero4();
        if (op != kOpXorOnly && nseg == 1) {
            acc = __ldcg(&L.partials[R.seg_first]);
        } else if (op != kOpXorOnly) {
            const int e0 = 31 - __clz(static_cast<uint32_t>(SB));
            for (uint32_t e = tid; e < 5u * 512u; e += kThreads) gtab[e] = __ldg(&tab_pow2(S, e0 + static_cast<int>(e >> 9))[e & 511u]);
            __syncthreads();
            const uint32_t nchunk = (nseg + 31) / 32, first = nseg - (nchunk - 1) * 32;
            for (uint32_t c0 = 0; c0 < nchunk; c0 += kThreads) {
                const uint32_t round = nchunk - c0 < kThreads ? nchunk - c0 : kThreads;
                for (uint32_t c = c0 + warp; c < c0 + round; c += 8) {
                    const uint32_t cnt = c == 0 ? first : 32, start = c == 0 ? 0 : first + (c - 1) * 32;
                    const uint32_t pad = 32 - cnt;
                    uint4 v = lane >= pad ? __ldcg(&L.partials[R.seg_first + start + lane - pad]) : zero4();
#pragma unroll
                    for (int b = 0; b < 5; ++b) {
                        const uint4 left = shfl_up4(v, 1u << b);
                        const uint32_t grp = (2u << b) - 1u;
                        if ((lane & grp) == grp) v = xor4(gf_mul_table<1, false>(left, gtab + 512 * b, 0), v);
                    }
                    if (lane == 31) red[c - c0] = v;
                }
                __syncthreads();
                if (warp == 0) {
                    for (uint32_t c = 0; c < round; ++c)
                        acc = (c0 == 0 && c == 0) ? red[0] : xor4(gf_mul_warp<true>(acc, tab_pow2(S, e0 + 5), lane), red[c]);
                }
                __syncthreads();
            }
            if (w + gridDim.x < L.total_segs) {   // more segments for this CTA: restore the Horner table
                for (uint32_t i = tid; i < 4096; i += kThreads) gtab[i] = __ldg(&S->byte256[i]);
                __syncthreads();
            }
        }
        if (warp == 0) {
            if (lane == 0) {
                uint32_t ok = 1u;
                if (op == kOpDecrypt || op == kOpVerify || op == kOpEncrypt) {
                    const uint4 mask = aes128_encrypt_global(j0_block_le(R.iv), S->rk);
                    const uint4 tag = xor4(acc, mask);
                    if (op == kOpEncrypt) {
                        store_partial16(R.tag_out, tag, 16);
                    } else {
                        ok = equal4(tag, load_partial16(R.tag_in, 16)) ? 1u : 0u;
                        *R.status = ok;
                    }
                } else if (op == kOpGhash) {
                    uint4 tag = acc;
                    if (flags & kGhashFinalize) tag = xor4(tag, load_partial16(R.tag_mask, 16));
                    store_partial16(R.tag_out, tag, 16);
                    if (flags & kGhashVerify) ok = equal4(tag, load_partial16(R.tag_in, 16)) ? 1u : 0u;
                    if (R.status) *R.status = ok;
                } else if (R.status) {
                    *R.status = 1u;   // kOpXorOnly: profiling control, no authentication
                }
                s_ok = ok;
                L.counters[r] = 0u;
            }
        }
        __syncthreads();
        const bool gated = op == kOpDecrypt || (op == kOpGhash && (flags & kGhashXorOnSuccess));
        if (!s_ok && gated && out) {
            for (uint64_t off = static_cast<uint64_t>(tid) * 16u; off < count; off += 16u * kThreads)
                store_block(out + off, zero4(), count - off, aligned);
        }
    }
}

// ----------------------------------------------------------------------------
// Layer kernels: uniform records, descriptors in kernel parameters.
// ----------------------------------------------------------------------------
// Programmatic dependent launch.  The layer kernels are launched so that the
// next kernel in the stream may start once every CTA of the current one has
// passed launch_dependents (its CTAs then fill their shared-memory tables
// while this grid drains); grid_dependency_wait() returns when the previous
// grid has completed and its writes are visible.  Both are no-ops for a
// normal launch.  Every CTA of a layer grid is resident at once (grid <= one
// CTA per SM), so a dependent grid never waits on CTAs that cannot start.
__device__ __forceinline__ void allow_dependent_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void layer_iv(uint32_t iv0, uint64_t ticket, uint32_t iv[4])
{
    iv[0] = iv0;
    iv[1] = static_cast<uint32_t>(ticket >> 32);
    iv[2] = static_cast<uint32_t>(ticket);
    iv[3] = 2u;
}

// Counter-mode constants of one record (IV words iv[0..2], counters below
// 2^16).  After AddRoundKey 0 the state is s0..s2 = IV ^ rk, s3 = BE32(ctr) ^
// rk[3]; only bytes 14 and 15 of the counter change, and they reach round 1's
// columns 1 and 0 alone.  So round 1 is t0 = a0 ^ Te3[byte 15],
// t1 = a1 ^ Te2[byte 14], t2 = a2, t3 = a3, and round 2 needs the eight
// lookups of t0 and t1 beside the constants b0..b3 (Bernstein and Schwabe's
// counter-mode caching for table AES): 138 lookups per block instead of 160.
struct CtrCache {
    uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
};

__device__ __forceinline__ CtrCache ctr_cache(const uint32_t iv[4], const Aes4Tables& T, const uint32_t* __restrict__ rk)
{
    const uint32_t s0 = bswap32(iv[0]) ^ rk[0], s1 = bswap32(iv[1]) ^ rk[1], s2 = bswap32(iv[2]) ^ rk[2];
    const uint32_t s3 = rk[3];   // counter bytes 12 and 13 are zero; 14 and 15 are looked up per block
    CtrCache K;
    K.a0 = T.look(0, s0, 0) ^ T.look(1, s1, 1) ^ T.look(2, s2, 2) ^ rk[4];
    K.a1 = T.look(0, s1, 0) ^ T.look(1, s2, 1) ^ T.look(3, s0, 3) ^ rk[5];
    K.a2 = T.look(0, s2, 0) ^ T.look(1, s3, 1) ^ T.look(2, s0, 2) ^ T.look(3, s1, 3) ^ rk[6];
    K.a3 = T.look(0, s3, 0) ^ T.look(1, s0, 1) ^ T.look(2, s1, 2) ^ T.look(3, s2, 3) ^ rk[7];
    K.b0 = T.look(2, K.a2, 2) ^ T.look(3, K.a3, 3) ^ rk[8];
    K.b1 = T.look(1, K.a2, 1) ^ T.look(2, K.a3, 2) ^ rk[9];
    K.b2 = T.look(0, K.a2, 0) ^ T.look(1, K.a3, 1) ^ rk[10];
    K.b3 = T.look(0, K.a3, 0) ^ T.look(3, K.a2, 3) ^ rk[11];
    return K;
}

// E_K(IV || BE32(ctr)) for ctr < 2^16 from the record's constants.
__device__ __forceinline__ uint4 aes128_ctr_cached(uint32_t ctr, const CtrCache& K, const Aes4Tables& T,
                                                   const uint32_t* __restrict__ rk)
{
    const uint32_t s3 = bswap32(ctr) ^ rk[3];
    const uint32_t t0 = K.a0 ^ T.look(3, s3, 3), t1 = K.a1 ^ T.look(2, s3, 2);
    uint32_t s[4] = {K.b0 ^ T.look(0, t0, 0) ^ T.look(1, t1, 1), K.b1 ^ T.look(0, t1, 0) ^ T.look(3, t0, 3),
                     K.b2 ^ T.look(2, t0, 2) ^ T.look(3, t1, 3), K.b3 ^ T.look(1, t0, 1) ^ T.look(2, t1, 2)};
    return aes128_rounds_from(make_uint4(s[0], s[1], s[2], s[3]), 3, T, rk);
}

// Keystream of every record plus E_K(J0) in the record's last 16 bytes.
// Each CTA takes one contiguous range of the layer's (record, block) space and
// its threads stride through it, so a thread meets at most a few records and
// derives each record's counter-mode constants once.
template <int kCap>
__global__ void __launch_bounds__(kLayerCtrThreads, 1) gcm_layer_ctr_kernel(const __grid_constant__ LayerLaunch<kCap> L)
{
    extern __shared__ __align__(16) uint8_t smem[];
    fill_aes4_smem(smem, L.h.sched);
    __syncthreads();
    // The keystream buffer may still be read by the previous verify grid.
    allow_dependent_launch();
    grid_dependency_wait();
    // Round keys in registers: the lookups are the kernel's only shared loads.
    uint32_t rk[44];
#pragma unroll
    for (int i = 0; i < 44; ++i) rk[i] = reinterpret_cast<const uint32_t*>(smem + kCtrTableBytes)[i];
    const Aes4Tables T = aes4_view(smem);
    const uint32_t payload_blocks = static_cast<uint32_t>((L.h.count + 15) >> 4);
    const uint32_t nb = payload_blocks + 1;
    const uint32_t total = nb * L.h.n;
    // Counters 2 .. payload_blocks + 1 (and 1 for J0) below 2^16: cached rounds.
    const bool cached = payload_blocks + 2u <= 65536u;
    const uint32_t per_cta = (total + gridDim.x - 1) / gridDim.x;
    const uint32_t beg = blockIdx.x * per_cta;
    const uint32_t end = beg + per_cta < total ? beg + per_cta : total;
    // (record, block) of the thread's position, advanced without a division.
    uint32_t gb = beg + threadIdx.x;
    uint32_t r = gb / nb, c = gb - r * nb;
    uint32_t cur = ~0u;
    uint32_t iv[4] = {0, 0, 0, 0};
    CtrCache K{};
    for (; gb < end; gb += blockDim.x) {
        if (r != cur) {
            layer_iv(L.h.iv0, L.rec[r].ticket, iv);
            if (cached) K = ctr_cache(iv, T, rk);
            cur = r;
        }
        uint8_t* out = L.h.ks + static_cast<uint64_t>(r) * L.h.ks_stride + 16ull * c;
        uint4 ks;
        if (cached) {
            ks = aes128_ctr_cached(c == payload_blocks ? 1u : 2u + c, K, T, rk);
        } else {
            const uint4 in = c == payload_blocks ? j0_block_le(iv) : ctr_block_le(iv, c);
            ks = aes128_encrypt_t4(in, T, rk);
        }
        if (L.h.unaligned) store_partial16(out, ks, 16); else *reinterpret_cast<uint4*>(out) = ks;
        c += blockDim.x;
        while (c >= nb) {
            c -= nb;
            ++r;
        }
    }
}

// The same keystream (and E_K(J0) in each record's last 16 bytes) from the
// bitsliced AES of bitsliced_aes.cuh: no table lookups, only integer logic
// (the S-box circuit, MixColumns XORs, a bit transpose per output word).  A
// thread takes one counter group of a record, v = 32 g .. 32 g + 31 (v = 1 is
// J0, payload block c has v = c + 2, v = 0 is not used); the round keys become
// plane masks in shared memory once per CTA.  It exists to be measured
// against the T-table kernel (SECURE_INFER_AES_KEYSTREAM=bitsliced selects it).
constexpr uint32_t kBsThreads = 256;

template <int kCap>
__global__ void __launch_bounds__(kBsThreads, 1) gcm_layer_ctr_bs_kernel(const __grid_constant__ LayerLaunch<kCap> L)
{
    __shared__ __align__(16) uint32_t mask[1408];
    for (uint32_t i = threadIdx.x; i < 1408u; i += blockDim.x) {
        const uint32_t b = i >> 3, k = i & 7u;
        const uint32_t byte = (L.h.sched->rk[b >> 2] >> (8u * (b & 3u))) & 0xffu;
        mask[i] = ((byte >> (7u - k)) & 1u) ? 0xffffffffu : 0u;
    }
    __syncthreads();
    // The keystream buffer may still be read by the previous verify grid.
    allow_dependent_launch();
    grid_dependency_wait();
    const uint32_t payload_blocks = static_cast<uint32_t>((L.h.count + 15) >> 4);
    const uint32_t groups = (payload_blocks + 2u + 31u) / 32u;
    const uint32_t total = groups * L.h.n;
    for (uint32_t item = blockIdx.x * blockDim.x + threadIdx.x; item < total; item += gridDim.x * blockDim.x) {
        const uint32_t r = item / groups, g = item - r * groups;
        const uint64_t ticket = L.rec[r].ticket;
        const uint32_t iv[3] = {L.h.iv0, static_cast<uint32_t>(ticket >> 32), static_cast<uint32_t>(ticket)};
        uint32_t st[16][8];
        bs_load_group(st, iv, g, mask);
        bs_encrypt(st, mask);
        uint8_t* rec = L.h.ks + static_cast<uint64_t>(r) * L.h.ks_stride;
        // Each output word goes out as soon as it is transposed, so only 32
        // of its words are live beside the remaining planes.
        auto store_word = [&](const uint32_t (&w)[32], int word) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const uint32_t v = 32u * g + static_cast<uint32_t>(j);
                if (v == 0u || (v >= 2u && v - 2u >= payload_blocks)) continue;
                uint8_t* out = (v == 1u ? rec + (L.h.ks_stride - 16) : rec + 16ull * (v - 2u)) + 4 * word;
                if (L.h.unaligned) store_partial16(out, make_uint4(w[j], 0, 0, 0), 4);
                else *reinterpret_cast<uint32_t*>(out) = w[j];
            }
        };
        {
            uint32_t w[32];
            bs_store_word<0>(st, w);
            store_word(w, 0);
        }
        {
            uint32_t w[32];
            bs_store_word<1>(st, w);
            store_word(w, 1);
        }
        {
            uint32_t w[32];
            bs_store_word<2>(st, w);
            store_word(w, 2);
        }
        {
            uint32_t w[32];
            bs_store_word<3>(st, w);
            store_word(w, 3);
        }
    }
}

// Fused verify + XOR + scatter.  One CTA of 8 warps per SM; each warp takes
// one segment of 32 k blocks (k <= 64, chosen per launch so the segments fill
// the warps once) of X = AAD || payload || len, aligned to the END of X (the
// first segment takes the shorter remainder).  Lane l = 8 q + r hashes blocks
// base + l + 32 j with Horner stride H^32 (8x-replicated shared table),
// prefetching four steps ahead.  The segment partial
//   sum_l Y_l H^(32 - l),  32 - l = (8 - r) + (24 - 8 q)
// is formed in shared memory: every lane scales by H^(8 - r) (eight tables
// interleaved like replicas, so a quarter-warp is conflict-free), quarters
// XOR-reduce and scale by H^(24 - 8 q), then the quarters XOR-reduce.  The
// last warp of a record joins the partials with H^(32 k), XORs the tag mask
// the keystream kernel left behind, compares, writes the status and zeroes
// the record's output on a mismatch ("write then gate").
enum : int { kLayerVerifyRaw = 0, kLayerVerifyCodec8 = 1, kLayerEncrypt = 2, kLayerVerifyCodec4 = 3 };
// Threads per verify/encrypt CTA: one CTA per SM shares the tables.  Raw
// verify and encrypt fit 128 registers, so 16 warps cover load and ALU
// latency; the codec modes need more registers and run 8 warps.
__host__ __device__ constexpr uint32_t layer_threads(int mode)
{
    return mode == kLayerVerifyRaw || mode == kLayerEncrypt ? 512u : 256u;
}
// byte32 (64 KiB), lane8 (64 KiB), H^8/16/24 (24 KiB), the segment join
// tables H^(32 S 2^b) for b = 0..4 (40 KiB).
constexpr size_t kLayerSmem = 2 * kGhashSmem + 8 * 512 * sizeof(uint4);
constexpr int kLayerPrefetch = 2;

// Decrypted fp32 parameters (scale or low) of a codec packet: N consecutive
// words at byte `off`, each C ^ KS (16-byte aligned).
template <int N>
__device__ __forceinline__ void load_params(const uint8_t* in, const uint8_t* ks, uint64_t off, float (&v)[32])
{
#pragma unroll
    for (int k = 0; k < N; k += 4) {
        const uint4 c = ldg16(in + off + 4 * k), m = ldg16(ks + off + 4 * k);
        v[k] = __uint_as_float(c.x ^ m.x);
        v[k + 1] = __uint_as_float(c.y ^ m.y);
        v[k + 2] = __uint_as_float(c.z ^ m.z);
        v[k + 3] = __uint_as_float(c.w ^ m.w);
    }
}

// One 16-byte block of quantised bytes (16 int8 or 32 int4 elements) of
// packet block c -> bf16 at out + 2 e0: v = fp32(q * scale) then fp32(v + low),
// round-to-nearest-even bf16 (optimized_decode.py:18-25).  For K (64-token
// groups per channel) the lane's 16/32 consecutive channel parameters are
// kept in registers, keyed by their first index, and reloaded only when the
// token group or channel set changes.
template <int N>
__device__ __forceinline__ void layer_dequant(uint4 p, uint64_t c, const CodecParams& cp, uint32_t kind,
                                              const uint8_t* in, const uint8_t* ksp, uint8_t* out, uint32_t& key,
                                              float (&sc)[32], float (&lo)[32])
{
    // q -> fp32 without the conversion unit: a byte permute places q in the
    // low mantissa byte of 2^23 (0x4B000000), and subtracting 2^23 is exact.
    constexpr uint32_t kTwo23 = 0x4B000000u;
    const uint32_t w[4] = {p.x, p.y, p.z, p.w};
    float q[N];
    if constexpr (N == 16) {
#pragma unroll
        for (int k = 0; k < 16; ++k)
            q[k] = __fsub_rn(__uint_as_float(__byte_perm(w[k >> 2], kTwo23, 0x7650u | (k & 3))), 8388608.0f);
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t lo4 = w[j] & 0x0f0f0f0fu, hi4 = (w[j] >> 4) & 0x0f0f0f0fu;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                q[8 * j + 2 * b] = __fsub_rn(__uint_as_float(__byte_perm(lo4, kTwo23, 0x7650u | b)), 8388608.0f);
                q[8 * j + 2 * b + 1] = __fsub_rn(__uint_as_float(__byte_perm(hi4, kTwo23, 0x7650u | b)), 8388608.0f);
            }
        }
    }
    const uint32_t e0 = static_cast<uint32_t>(c) * N;
    float v[N];
    if (kind == 0) {
        const uint32_t hd = cp.heads * 128u;
        const uint32_t sidx0 = (e0 / (64u * hd)) * hd + (e0 % hd);
        if (sidx0 != key) {
            load_params<N>(in, ksp, cp.qb + 4ull * sidx0, sc);
            load_params<N>(in, ksp, cp.qb + cp.sb + 4ull * sidx0, lo);
            key = sidx0;
        }
#pragma unroll
        for (int k = 0; k < N; ++k) v[k] = __fadd_rn(__fmul_rn(q[k], sc[k]), lo[k]);
    } else {
        const uint64_t so = cp.qb + 4ull * (e0 / 64u), lo_off = so + cp.sb;
        const float s1 = __uint_as_float(__ldg(reinterpret_cast<const uint32_t*>(in + so)) ^
                                         __ldg(reinterpret_cast<const uint32_t*>(ksp + so)));
        const float l1 = __uint_as_float(__ldg(reinterpret_cast<const uint32_t*>(in + lo_off)) ^
                                         __ldg(reinterpret_cast<const uint32_t*>(ksp + lo_off)));
#pragma unroll
        for (int k = 0; k < N; ++k) v[k] = __fadd_rn(__fmul_rn(q[k], s1), l1);
    }
    uint4* dst = reinterpret_cast<uint4*>(out + 2u * static_cast<size_t>(e0));
#pragma unroll
    for (int k = 0; k < N; k += 8) {
        uint4 o;
        __nv_bfloat162 b;
        b = __floats2bfloat162_rn(v[k + 0], v[k + 1]); o.x = *reinterpret_cast<uint32_t*>(&b);
        b = __floats2bfloat162_rn(v[k + 2], v[k + 3]); o.y = *reinterpret_cast<uint32_t*>(&b);
        b = __floats2bfloat162_rn(v[k + 4], v[k + 5]); o.z = *reinterpret_cast<uint32_t*>(&b);
        b = __floats2bfloat162_rn(v[k + 6], v[k + 7]); o.w = *reinterpret_cast<uint32_t*>(&b);
        dst[k / 8] = o;
    }
}

// Publishes a warp's segment partial and counts it; true in the warp that
// completes record r.  The warp's output stores are ordered before the count
// by the warp barrier and one device-scope fence in lane 0 (the ordering the
// fail-closed zeroing of the completing warp relies on), and that warp's lane
// 0 fences again before its lanes read the other partials.
__device__ __forceinline__ bool publish_partial(uint4* partials, uint32_t* counters, uint32_t w, uint32_t r,
                                                uint32_t nseg, uint4 part, uint32_t lane)
{
    __syncwarp();
    uint32_t last = 0;
    if (lane == 0) {
        partials[w] = part;
        __threadfence();
        last = atomicAdd(&counters[r], 1u) == nseg - 1 ? 1u : 0u;
        if (last) __threadfence();
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    __syncwarp();
    return last != 0;
}

template <int kCap, int kMode>
__global__ void __launch_bounds__(layer_threads(kMode), 1) gcm_layer_verify_kernel(const __grid_constant__ LayerLaunch<kCap> L)
{
    constexpr bool kCodec = kMode == kLayerVerifyCodec8 || kMode == kLayerVerifyCodec4;
    constexpr bool kEncrypt = kMode == kLayerEncrypt;
    extern __shared__ __align__(16) uint8_t smem[];
    uint4* gtab = reinterpret_cast<uint4*>(smem);
    uint4* ltab = reinterpret_cast<uint4*>(smem + kGhashSmem);
    uint4* qtab = reinterpret_cast<uint4*>(smem + 2 * kGhashSmem);   // [3][512]: H^8, H^16, H^24
    uint4* jtab = qtab + 3 * 512;                                    // [5][512]: H^(32 S 2^b), b = 0..4
    const GcmSchedule* __restrict__ S = L.h.sched;
    const uint32_t tid = threadIdx.x, lane = tid & 31u, rep = lane & 7u, quarter = lane >> 3;
    const uint32_t seg_steps = L.h.seg_steps;
    __shared__ __align__(8) uint64_t tables_bar, gtab_bar;
    // Tables used only after a warp's main loop (lane, quarter and join
    // tables, 128 KiB) stream in by bulk copy while the main loop runs.
    if (tid == 0) {
        // The Horner multiplier H^32 as byte tables (64 KiB), needed from the
        // first step on; waited for after each warp has issued its first loads.
        mbar_init_expect(&gtab_bar, 65536u);
        bulk_g2s(gtab, S->byte32, 65536u, &gtab_bar);
        mbar_init_expect(&tables_bar, 65536u + 8u * 8192u);
        bulk_g2s(ltab, S->lane8, 65536u, &tables_bar);
        bulk_g2s(qtab, S->tab[tab_pow_small(8)], 8192u, &tables_bar);
        bulk_g2s(qtab + 512, S->tab[tab_pow_small(16)], 8192u, &tables_bar);
        bulk_g2s(qtab + 1024, S->tab[tab_pow_small(24)], 8192u, &tables_bar);
        bulk_g2s(jtab, S->tab[tab_pow_32k(seg_steps)], 8192u, &tables_bar);
        bulk_g2s(jtab + 512, L.h.join_pow, 4u * 8192u, &tables_bar);
    }
    constexpr uint32_t kLayerThreads = layer_threads(kMode), kLayerWarps = kLayerThreads / 32;
    __syncthreads();
    // Records, keystream and destinations are touched only after the
    // previous grid (the keystream kernel) has completed.
    allow_dependent_launch();
    grid_dependency_wait();
    bool tables_ready = false, gtab_ready = false;

    const uint64_t count = L.h.count;
    const bool aligned = L.h.unaligned == 0;
    const int64_t seg_blocks = 32 * static_cast<int64_t>(seg_steps);
    const int64_t a_blk = 4;   // 64-byte AAD
    const int64_t n_blk = static_cast<int64_t>((count + 15) >> 4);
    const int64_t m = a_blk + n_blk + 1;
    const uint32_t nseg = L.h.nseg;
    const int64_t len0 = m - static_cast<int64_t>(nseg - 1) * seg_blocks;
    const uint64_t tag_off = ((count + 31) & ~uint64_t(31)) ? ((count + 31) & ~uint64_t(31)) : 32;
    const uint32_t total = nseg * L.h.n;
    const uint4 len_blk = len_block_le(64, count);
    const CodecParams cp = L.h.codec;
    // On a tag mismatch the record's destination is zeroed: raw bytes, or the
    // whole bf16 block a codec packet decodes into.
    const uint64_t out_bytes = kCodec ? 2ull * 128u * cp.heads * 128u : count;

    for (uint32_t w = blockIdx.x + gridDim.x * (tid >> 5); w < total; w += gridDim.x * kLayerWarps) {
        const uint32_t r = w / nseg, k = w - r * nseg;
        // Verify: record -> plaintext destination.  Encrypt: plaintext
        // source -> record (C || tag || 0^16 || AAD).
        uint8_t* rec_ptr = const_cast<uint8_t*>(L.h.records) + static_cast<uint64_t>(r) * L.h.stride;
        const uint8_t* in = kEncrypt ? L.rec[r].dst : rec_ptr;
        const uint8_t* aad = kEncrypt ? L.h.aad + 64ull * r : rec_ptr + tag_off + 32;
        const uint8_t* ksp = L.h.ks + static_cast<uint64_t>(r) * L.h.ks_stride;
        uint8_t* out = kEncrypt ? rec_ptr : L.rec[r].dst;
        const int64_t seg_end = len0 + static_cast<int64_t>(k) * seg_blocks;
        const int64_t seg_len = k == 0 ? len0 : seg_blocks;
        const int J = static_cast<int>((seg_len + 31) / 32);
        const int64_t base = seg_end - static_cast<int64_t>(J) * 32;

        // Interior steps [j_lo, j_hi): every lane holds a full 16-byte
        // payload block of an aligned record, at byte offset off0 + 512 j.
        // They skip the per-lane AAD / length-block / tail checks.
        const int64_t n_full = aligned ? static_cast<int64_t>(count >> 4) : 0;
        const int64_t lo_num = a_blk - base, hi_num = a_blk + n_full - 32 - base;
        const int j_lo = lo_num <= 0 ? 0 : static_cast<int>((lo_num + 31) / 32);
        const int j_hi = hi_num < 0 ? 0 : (hi_num / 32 + 1 < J ? static_cast<int>(hi_num / 32 + 1) : J);
        const int64_t off0 = (base + lane - a_blk) * 16;
        auto interior = [&](int j) { return j >= j_lo && j < j_hi; };
        auto load = [&](int j, uint4& x, uint4& ks) {
            if (interior(j)) {
                const uint64_t off = static_cast<uint64_t>(off0 + 512ll * j);
                x = ldg16(in + off);
                ks = ldg16(ksp + off);
                return;
            }
            x = zero4();
            ks = zero4();
            const int64_t i = base + lane + 32 * static_cast<int64_t>(j);
            if (j >= J || i < 0) return;
            if (i < a_blk) {
                x = aligned ? ldg16(aad + 16 * i) : load_partial16(aad + 16 * i, 16);
            } else if (i < a_blk + n_blk) {
                const uint64_t off = static_cast<uint64_t>(i - a_blk) * 16u;
                const uint64_t avail = count - off;
                if (aligned && avail >= 16) {
                    x = ldg16(in + off);
                    ks = ldg16(ksp + off);
                } else {
                    x = load_partial16(in + off, avail);
                    ks = load_partial16(ksp + off, avail);
                }
            } else {
                x = len_blk;
            }
        };
        uint4 Y = zero4();            // Horner accumulator; 0 * H^32 = 0 starts it
        uint32_t pkey = ~0u;          // codec: index of the cached K parameters
        float psc[32], plo[32];
        const uint32_t kind = r >= L.h.v_first ? 1u : 0u;
        // Any step through the general path: AAD, payload, partial and
        // length blocks in any mix.
        auto consume = [&](int j, uint4 x0, uint4 k0) {
            const int64_t i = base + lane + 32 * static_cast<int64_t>(j);
            if (i >= a_blk && i < a_blk + n_blk) {
                const uint64_t off = static_cast<uint64_t>(i - a_blk) * 16u;
                if constexpr (kCodec) {
                    if (off < cp.qb)
                        layer_dequant<kMode == kLayerVerifyCodec8 ? 16 : 32>(xor4(x0, k0), off >> 4, cp, kind, in,
                                                                           ksp, out, pkey, psc, plo);
                } else if constexpr (kEncrypt) {
                    // C is zero past `count` (both loads are), so the whole
                    // block goes out: the record's padding must be zero.
                    store_block(out + off, xor4(x0, k0), 16, aligned);
                } else {
                    store_block(out + off, xor4(x0, k0), count - off, aligned);
                }
            }
            // GHASH runs over the ciphertext: loaded (verify) or just formed (encrypt).
            Y = xor4(gf_mul_byte8(Y, gtab, rep), kEncrypt ? xor4(x0, k0) : x0);
        };
        // Slot u of a prefetch ring holds step j0 + u and is refilled in
        // place with step j0 + u + kLayerPrefetch once consumed.  The inner
        // loops are unrolled so every slot keeps its own registers: moving a
        // register whose load is still in flight would wait for that load.
        uint4 xq[kLayerPrefetch], kq[kLayerPrefetch];
        if constexpr (kCodec) {
            // Codec packets: the warp's payload blocks (packets, scales and
            // lows) and their keystream stream into L2 first; the loop then
            // loads one step ahead and is not unrolled, so the large
            // dequantising body is emitted once.
            const int64_t i0 = base > a_blk ? base : a_blk;
            const int64_t i1 = seg_end < a_blk + n_blk ? seg_end : a_blk + n_blk;
            if (lane == 0 && i1 > i0) {
                const uint64_t off = static_cast<uint64_t>(i0 - a_blk) * 16u;
                l2_prefetch_bulk(in + off, static_cast<uint32_t>(i1 - i0) * 16u);
                l2_prefetch_bulk(ksp + off, static_cast<uint32_t>(i1 - i0) * 16u);
            }
            uint4 xc, kc;
            load(0, xc, kc);
            if (!gtab_ready) gtab_ready = mbar_wait_bounded(&gtab_bar, 0);
#pragma unroll 1
            for (int j = 0; j < J; ++j) {
                const uint4 x0 = xc, k0 = kc;
                load(j + 1, xc, kc);
                consume(j, x0, k0);
            }
        } else {
            // General head (AAD side), tight interior, general tail (length
            // block, partial last block).  Interior segments are all interior.
            const int lo = j_lo < J ? j_lo : J;
            const int hi = j_hi > lo ? j_hi : lo;
            // Encrypt: the warp's interior is one contiguous range of the
            // plaintext and of the keystream, streamed into L2 ahead of the
            // loads below.  Raw verify loads without it (measured 2 % faster
            // per c2 layer: the bulk requests of every warp at once queue
            // ahead of the first steps' loads).
            if (kEncrypt && lane == 0 && hi > lo) {
                const uint64_t off = static_cast<uint64_t>((base - a_blk) * 16 + 512ll * lo);
                const uint32_t bytes = static_cast<uint32_t>(hi - lo) * 512u;
                l2_prefetch_bulk(in + off, bytes);
                l2_prefetch_bulk(ksp + off, bytes);
            }
#pragma unroll
            for (int u = 0; u < kLayerPrefetch; ++u) {
                if (lo + u < hi) {
                    const uint64_t off = static_cast<uint64_t>(off0 + 512ll * (lo + u));
                    xq[u] = ldg16(in + off);
                    kq[u] = ldg16(ksp + off);
                }
            }
            if (!gtab_ready) gtab_ready = mbar_wait_bounded(&gtab_bar, 0);
#pragma unroll 1
            for (int j = 0; j < lo; ++j) {
                uint4 x0, k0;
                load(j, x0, k0);
                consume(j, x0, k0);
            }
#pragma unroll 1
            for (int j0 = lo; j0 < hi; j0 += kLayerPrefetch) {
#pragma unroll
                for (int u = 0; u < kLayerPrefetch; ++u) {
                    const int j = j0 + u;
                    if (j >= hi) break;
                    const uint4 x0 = xq[u], k0 = kq[u];
                    if (j + kLayerPrefetch < hi) {
                        const uint64_t nxt = static_cast<uint64_t>(off0 + 512ll * (j + kLayerPrefetch));
                        xq[u] = ldg16(in + nxt);
                        kq[u] = ldg16(ksp + nxt);
                    }
                    const uint4 c = xor4(x0, k0);
                    *reinterpret_cast<uint4*>(out + static_cast<uint64_t>(off0 + 512ll * j)) = c;
                    Y = xor4(gf_mul_byte8(Y, gtab, rep), kEncrypt ? c : x0);
                }
            }
#pragma unroll 1
            for (int j = hi; j < J; ++j) {
                uint4 x0, k0;
                load(j, x0, k0);
                consume(j, x0, k0);
            }
        }
        // Two-stage lane combine in shared memory.  If the table copy never
        // completes the partial is poisoned, so the record fails closed
        // (status 0, output zeroed) instead of waiting forever.
        if (!tables_ready) tables_ready = mbar_wait_bounded(&tables_bar, 0);
        if (!tables_ready || !gtab_ready) Y = make_uint4(~0u, ~0u, ~0u, ~0u);
        Y = gf_mul_table<8, false>(Y, ltab, rep);                       // * H^(8 - r)
        Y = xor4(Y, shfl_xor4(Y, 1));
        Y = xor4(Y, shfl_xor4(Y, 2));
        Y = xor4(Y, shfl_xor4(Y, 4));                                   // quarter sum
        {
            const uint4 Yq = gf_mul_quarter(Y, qtab + 512 * (quarter < 3 ? 2 - quarter : 0), rep, quarter != 3);
            if (quarter != 3) Y = Yq;                                    // * H^(24 - 8 q)
        }
        Y = xor4(Y, shfl_xor4(Y, 8));
        uint4 part = xor4(Y, shfl_xor4(Y, 16));
        // The record's GHASH is S = sum_k p_k H^(L (nseg - 1 - k)), L = 32
        // seg_steps blocks per segment.  With at most 64 segments each warp
        // scales its own partial by H^(L e), e = nseg - 1 - k, one warp-wide
        // product per set bit of e (tables H^(L 2^b), b = 0..5), so the warp
        // that completes the record only XORs the partials.
        const bool prescaled = nseg <= 64u;
        if (prescaled) {
            const uint32_t e = nseg - 1u - k;
#pragma unroll
            for (int b = 0; b < 5; ++b)
                if (e & (1u << b)) part = gf_mul_warp<false>(part, jtab + 512 * b, static_cast<int>(lane));
            if (e & 32u) part = gf_mul_warp<true>(part, L.h.join_pow + 4 * 512, static_cast<int>(lane));
        }

        // The record's tag, loaded before the count so that the warp that
        // completes the record does not wait for it afterwards.
        const uint4 tag_in = kEncrypt ? zero4() : load_partial16(in + tag_off, 16);
        if (!publish_partial(L.h.partials, L.h.counters, w, r, nseg, part, lane)) continue;
        uint4 acc = zero4();
        if (prescaled) {
            uint4 v = zero4();
            for (uint32_t i = lane; i < nseg; i += 32) v = xor4(v, __ldcg(&L.h.partials[r * nseg + i]));
            acc = warp_xor_reduce(v);
        }
        // Otherwise join the partials here: chunks of 32 partials (the first
        // chunk takes the remainder), each reduced by a tree over the lanes
        // (level b combines pairs of 2^b-partial groups with H^(L 2^b)),
        // chunks joined by Horner with H^(32 L).
        const uint32_t first = nseg - (nseg - 1) / 32 * 32;
        for (uint32_t k0 = 0; !prescaled && k0 < nseg;) {
            const uint32_t cnt = k0 == 0 ? first : 32;
            const uint32_t pad = 32 - cnt;     // zero partials in front keep the powers aligned
            uint4 v = lane >= pad ? __ldcg(&L.h.partials[r * nseg + k0 + lane - pad]) : zero4();
#pragma unroll
            for (int b = 0; b < 5; ++b) {
                const uint4 left = shfl_up4(v, 1u << b);
                const uint32_t grp = (2u << b) - 1u;
                if ((lane & grp) == grp) v = xor4(gf_mul_table<1, false>(left, jtab + 512 * b, 0), v);
            }
            v = make_uint4(__shfl_sync(0xffffffffu, v.x, 31), __shfl_sync(0xffffffffu, v.y, 31),
                           __shfl_sync(0xffffffffu, v.z, 31), __shfl_sync(0xffffffffu, v.w, 31));
            acc = k0 == 0 ? v : xor4(gf_mul_warp<true>(acc, L.h.join_pow + 4 * 512, lane), v);
            k0 += cnt;
        }
        const uint4 mask = *reinterpret_cast<const uint4*>(ksp + (L.h.ks_stride - 16));
        if constexpr (kEncrypt) {
            // tag, zero block, AAD copy, and zeros over [round16(count), tag_off).
            const uint64_t pad_first = (count + 15) & ~uint64_t(15);
            if (lane == 0) store_block(out + tag_off, xor4(acc, mask), 16, aligned);
            if (lane == 1) store_block(out + tag_off + 16, zero4(), 16, aligned);
            if (lane >= 2 && lane < 6)
                store_block(out + tag_off + 16 * lane, load_partial16(aad + 16 * (lane - 2), 16), 16, aligned);
            if (lane == 6 && pad_first < tag_off) store_block(out + pad_first, zero4(), 16, aligned);
            if (lane == 0) {
                L.h.status[r] = 1u;
                L.h.counters[r] = 0u;
            }
            continue;
        }
        const bool ok = equal4(xor4(acc, mask), tag_in);
        if (lane == 0) {
            L.h.status[r] = ok ? 1u : 0u;
            L.h.counters[r] = 0u;
        }
        if (!ok) {
            for (uint64_t off = static_cast<uint64_t>(lane) * 16u; off < out_bytes; off += 512u)
                store_block(out + off, zero4(), out_bytes - off, aligned);
        }
    }
}

// Fused verify with the keystream computed inside the kernel, for raw,
// 16-byte aligned records already in device memory (nothing to overlap a
// keystream prefetch with).  During the main loop shared memory holds what
// the loop reads: the four AES T-table replicas and round keys (128 KiB, as
// the keystream kernel) and the H^32 byte tables (64 KiB).  Segments and lanes
// are those of gcm_layer_verify_kernel.  An interior step of a warp loads 16
// bytes of ciphertext per lane two steps ahead, encrypts the lane's counter
// block (with the record's counter-mode constants, as the keystream kernel),
// XORs, stores and takes one Horner step; the AES lookups of one warp fill
// the load latency of the others, and no keystream crosses HBM.
//
// When every warp holds at most one segment and a record has at most 64 of
// them (the usual layer), the launch is a single pass: once all warps of the
// CTA are through their main loops, the lane, quarter and join tables (128
// KiB) replace the T-tables by one bulk copy, so the segment combine runs on
// conflict-free shared-memory tables as in gcm_layer_verify_kernel, and the
// first warp of each record folds E_K(J0) into its partial, so the XOR of a
// record's partials is its tag.  Otherwise (longer layers) each warp combines
// its segments through L1 from the schedule and the warp that completes a
// record computes E_K(J0) itself.
static_assert(offsetof(GcmSchedule, rk) == 0, "the host copies the round keys from the schedule's start");
constexpr uint32_t kInlineThreads = 512;
constexpr size_t kInlineSmem = kCtrTableBytes + 256 + kGhashSmem;
static_assert(kCtrTableBytes == 2 * kGhashSmem, "the combine tables take the T-tables' place");

template <int kCap>
__global__ void __launch_bounds__(kInlineThreads, 1)
    gcm_layer_verify_inline_kernel(const __grid_constant__ LayerLaunch<kCap> L)
{
    extern __shared__ __align__(16) uint8_t smem[];
    uint4* gtab = reinterpret_cast<uint4*>(smem + kCtrTableBytes + 256);
    // Single pass, after the main loops: the combine tables in the T-tables'
    // place (lane8 64 KiB, H^8/16/24 24 KiB, H^(L 2^b) for b = 0..4 40 KiB).
    uint4* ltab = reinterpret_cast<uint4*>(smem);
    uint4* qtab = reinterpret_cast<uint4*>(smem + kGhashSmem);
    uint4* jtab = qtab + 3 * 512;
    const GcmSchedule* __restrict__ S = L.h.sched;
    const uint32_t tid = threadIdx.x, lane = tid & 31u, rep = lane & 7u, quarter = lane >> 3;
    const uint32_t seg_steps = L.h.seg_steps;
    __shared__ __align__(8) uint64_t gtab_bar, comb_bar;
    if (tid == 0) {
        mbar_init_expect(&gtab_bar, 65536u);
        bulk_g2s(gtab, S->byte32, 65536u, &gtab_bar);
    }
    fill_aes4_smem(smem, S);
    __syncthreads();
    // Records and destinations are touched only after the previous grid in
    // the stream has completed.
    allow_dependent_launch();
    grid_dependency_wait();
    // If a table copy never completes, the partials are poisoned and the
    // records fail closed (status 0, output zeroed) instead of hanging.
    const bool gtab_ready = mbar_wait_bounded(&gtab_bar, 0);
    const uint32_t* rk = L.h.rk;   // constant bank
    const uint32_t* rk_smem = reinterpret_cast<const uint32_t*>(smem + kCtrTableBytes);   // for the AES calls
    const Aes4Tables T = aes4_view(smem);

    const uint64_t count = L.h.count;
    const int64_t seg_blocks = 32 * static_cast<int64_t>(seg_steps);
    const int64_t a_blk = 4;   // 64-byte AAD
    const int64_t n_blk = static_cast<int64_t>((count + 15) >> 4);
    const int64_t m = a_blk + n_blk + 1;
    const uint32_t nseg = L.h.nseg;
    const int64_t len0 = m - static_cast<int64_t>(nseg - 1) * seg_blocks;
    const uint64_t tag_off = ((count + 31) & ~uint64_t(31)) ? ((count + 31) & ~uint64_t(31)) : 32;
    const uint32_t total = nseg * L.h.n;
    const uint4 len_blk = len_block_le(64, count);
    constexpr uint32_t kWarps = kInlineThreads / 32;
    constexpr int kPf = 2;
    const bool cached = n_blk + 2 <= 65536;

    // Horner partial of segment k of record r (lane l: blocks base + l + 32 j,
    // stride H^32), with the record's plaintext written out.
    auto hash_segment = [&](uint32_t r, uint32_t k) -> uint4 {
        const uint8_t* in = L.h.records + static_cast<uint64_t>(r) * L.h.stride;
        const uint8_t* aad = in + tag_off + 32;
        uint8_t* out = L.rec[r].dst;
        uint32_t iv[4];
        layer_iv(L.h.iv0, L.rec[r].ticket, iv);
        // Counter-mode constants of the record (counters below 2^16).
        const CtrCache K = cached ? ctr_cache(iv, T, rk) : CtrCache{};
        const int64_t seg_end = len0 + static_cast<int64_t>(k) * seg_blocks;
        const int64_t seg_len = k == 0 ? len0 : seg_blocks;
        const int J = static_cast<int>((seg_len + 31) / 32);
        const int64_t base = seg_end - static_cast<int64_t>(J) * 32;
        // Interior steps [lo, hi): every lane on a full payload block.
        const int64_t n_full = static_cast<int64_t>(count >> 4);
        const int64_t lo_num = a_blk - base, hi_num = a_blk + n_full - 32 - base;
        const int j_lo = lo_num <= 0 ? 0 : static_cast<int>((lo_num + 31) / 32);
        const int j_hi = hi_num < 0 ? 0 : (hi_num / 32 + 1 < J ? static_cast<int>(hi_num / 32 + 1) : J);
        const int lo = j_lo < J ? j_lo : J;
        const int hi = j_hi > lo ? j_hi : lo;
        const int64_t c0 = base + lane - a_blk;   // payload block of step 0 (negative on the AAD)
        uint4 Y = zero4();
        uint4 xq[kPf];
#pragma unroll
        for (int u = 0; u < kPf; ++u)
            if (lo + u < hi) xq[u] = ldg16(in + static_cast<uint64_t>(c0 + 32ll * (lo + u)) * 16u);
        // Steps outside [lo, hi) take the general path (AAD, payload, partial
        // and length blocks in any mix, AES by call); the interior runs the
        // unrolled loop.
#pragma unroll 1
        for (int j = 0; j < J; ++j) {
            if (j == lo && lo < hi) {
#pragma unroll 1
                for (int j0 = lo; j0 < hi; j0 += kPf) {
#pragma unroll
                    for (int u = 0; u < kPf; ++u) {
                        const int jj = j0 + u;
                        if (jj >= hi) break;
                        const uint4 x0 = xq[u];
                        if (jj + kPf < hi) xq[u] = ldg16(in + static_cast<uint64_t>(c0 + 32ll * (jj + kPf)) * 16u);
                        const uint64_t c = static_cast<uint64_t>(c0 + 32ll * jj);
                        const uint4 ks = cached ? aes128_ctr_cached(2u + static_cast<uint32_t>(c), K, T, rk)
                                                : aes128_encrypt_t4(ctr_block_le(iv, c), T, rk);
                        *reinterpret_cast<uint4*>(out + c * 16u) = xor4(x0, ks);
                        Y = xor4(gf_mul_byte8(Y, gtab, rep), x0);
                    }
                }
                j = hi - 1;
                continue;
            }
            const int64_t i = base + lane + 32 * static_cast<int64_t>(j);
            uint4 x = zero4();
            if (i >= 0) {
                if (i < a_blk) {
                    x = ldg16(aad + 16 * i);
                } else if (i < a_blk + n_blk) {
                    const uint64_t off = static_cast<uint64_t>(i - a_blk) * 16u;
                    const uint64_t avail = count - off;
                    x = avail >= 16 ? ldg16(in + off) : load_partial16(in + off, avail);
                    const uint4 ks = aes128_encrypt_t4_call(ctr_block_le(iv, static_cast<uint64_t>(i - a_blk)), T, rk_smem);
                    store_block(out + off, xor4(x, ks), avail, true);
                } else {
                    x = len_blk;
                }
            }
            Y = xor4(gf_mul_byte8(Y, gtab, rep), x);
        }
        if (!gtab_ready) Y = make_uint4(~0u, ~0u, ~0u, ~0u);
        return Y;
    };

    // Tag check of record r by the warp that completed it: status, and on a
    // mismatch the record's plaintext zeroed.
    auto finish_record = [&](uint32_t r, uint4 tag, uint4 tag_in) {
        const bool ok = equal4(tag, tag_in);
        if (lane == 0) {
            L.h.status[r] = ok ? 1u : 0u;
            L.h.counters[r] = 0u;
        }
        if (!ok) {
            uint8_t* out = L.rec[r].dst;
            for (uint64_t off = static_cast<uint64_t>(lane) * 16u; off < count; off += 512u)
                store_block(out + off, zero4(), count - off, true);
        }
    };

    const bool single = total <= gridDim.x * kWarps && nseg <= 64u;
    for (uint32_t w = blockIdx.x + gridDim.x * (tid >> 5);; w += gridDim.x * kWarps) {
        const bool has = w < total;
        if (!single && !has) return;
        const uint32_t r = has ? w / nseg : 0u, k = has ? w - r * nseg : 0u;
        uint4 Y = zero4(), mask = zero4();
        uint32_t iv[4];
        layer_iv(L.h.iv0, has ? L.rec[r].ticket : 0ull, iv);
        if (has) Y = hash_segment(r, k);
        if (has && (!single || k == 0)) mask = aes128_encrypt_t4_call(j0_block_le(iv), T, rk_smem);
        if (single) {
            // Every warp of the CTA is through its T-table lookups.
            __syncthreads();
            if (tid == 0) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_init_expect(&comb_bar, 65536u + 8u * 8192u);
                bulk_g2s(ltab, S->lane8, 65536u, &comb_bar);
                bulk_g2s(qtab, S->tab[tab_pow_small(8)], 8192u, &comb_bar);
                bulk_g2s(qtab + 512, S->tab[tab_pow_small(16)], 8192u, &comb_bar);
                bulk_g2s(qtab + 1024, S->tab[tab_pow_small(24)], 8192u, &comb_bar);
                bulk_g2s(jtab, S->tab[tab_pow_32k(static_cast<int>(seg_steps))], 8192u, &comb_bar);
                bulk_g2s(jtab + 512, L.h.join_pow, 4u * 8192u, &comb_bar);
            }
            __syncthreads();
            const bool comb_ready = mbar_wait_bounded(&comb_bar, 0);
            if (!has) return;
            if (!comb_ready) Y = make_uint4(~0u, ~0u, ~0u, ~0u);
            Y = gf_mul_table<8, false>(Y, ltab, rep);                       // * H^(8 - r)
            Y = xor4(Y, shfl_xor4(Y, 1));
            Y = xor4(Y, shfl_xor4(Y, 2));
            Y = xor4(Y, shfl_xor4(Y, 4));                                   // quarter sum
            {
                const uint4 Yq = gf_mul_quarter(Y, qtab + 512 * (quarter < 3 ? 2 - quarter : 0), rep, quarter != 3);
                if (quarter != 3) Y = Yq;                                    // * H^(24 - 8 q)
            }
            Y = xor4(Y, shfl_xor4(Y, 8));
            uint4 part = xor4(Y, shfl_xor4(Y, 16));
            // Pre-scaled by H^(L e), e = nseg - 1 - k; segment 0 adds E_K(J0),
            // so the XOR of the record's partials is its tag.
            const uint32_t e = nseg - 1u - k;
#pragma unroll
            for (int b = 0; b < 5; ++b)
                if (e & (1u << b)) part = gf_mul_warp<false>(part, jtab + 512 * b, static_cast<int>(lane));
            if (e & 32u) part = gf_mul_warp<true>(part, L.h.join_pow + 4 * 512, static_cast<int>(lane));
            part = xor4(part, mask);
            const uint4 tag_in = ldg16(L.h.records + static_cast<uint64_t>(r) * L.h.stride + tag_off);
            if (!publish_partial(L.h.partials, L.h.counters, w, r, nseg, part, lane)) return;
            uint4 v = zero4();
            for (uint32_t i = lane; i < nseg; i += 32) v = xor4(v, __ldcg(&L.h.partials[r * nseg + i]));
            finish_record(r, warp_xor_reduce(v), tag_in);
            return;
        }
        // Several segments per warp: two-stage lane combine with the tables
        // read through L1.
        Y = gf_mul_table<8, true>(Y, S->lane8, rep);                    // * H^(8 - r)
        Y = xor4(Y, shfl_xor4(Y, 1));
        Y = xor4(Y, shfl_xor4(Y, 2));
        Y = xor4(Y, shfl_xor4(Y, 4));                                   // quarter sum
        if (quarter != 3) Y = gf_mul_table<1, true>(Y, S->tab[tab_pow_small(8 * (3 - static_cast<int>(quarter)))], 0);
        Y = xor4(Y, shfl_xor4(Y, 8));
        uint4 part = xor4(Y, shfl_xor4(Y, 16));
        // Pre-scaled partials as in gcm_layer_verify_kernel (tables H^(L 2^b):
        // b = 0 from the schedule, b = 1..5 from the session join tables).
        const bool prescaled = nseg <= 64u;
        if (prescaled) {
            const uint32_t e = nseg - 1u - k;
            if (e & 1u) part = gf_mul_warp<true>(part, S->tab[tab_pow_32k(static_cast<int>(seg_steps))], static_cast<int>(lane));
#pragma unroll
            for (int b = 1; b < 6; ++b)
                if (e & (1u << b)) part = gf_mul_warp<true>(part, L.h.join_pow + 512 * (b - 1), static_cast<int>(lane));
        }
        const uint4 tag_in = ldg16(L.h.records + static_cast<uint64_t>(r) * L.h.stride + tag_off);
        if (!publish_partial(L.h.partials, L.h.counters, w, r, nseg, part, lane)) continue;
        uint4 acc = zero4();
        if (prescaled) {
            uint4 v = zero4();
            for (uint32_t i = lane; i < nseg; i += 32) v = xor4(v, __ldcg(&L.h.partials[r * nseg + i]));
            acc = warp_xor_reduce(v);
        }
        // Otherwise join the record's partials as gcm_layer_verify_kernel does:
        // level b of the lane tree multiplies by H^(L 2^b) (b = 0 from the
        // schedule, b = 1..4 from the session join tables), chunks of 32 by
        // H^(32 L).
        const uint32_t first = nseg - (nseg - 1) / 32 * 32;
        for (uint32_t k0 = 0; !prescaled && k0 < nseg;) {
            const uint32_t cnt = k0 == 0 ? first : 32;
            const uint32_t pad = 32 - cnt;
            uint4 v = lane >= pad ? __ldcg(&L.h.partials[r * nseg + k0 + lane - pad]) : zero4();
#pragma unroll
            for (int b = 0; b < 5; ++b) {
                const uint4 left = shfl_up4(v, 1u << b);
                const uint32_t grp = (2u << b) - 1u;
                const uint4* tb = b == 0 ? S->tab[tab_pow_32k(static_cast<int>(seg_steps))] : L.h.join_pow + 512 * (b - 1);
                if ((lane & grp) == grp) v = xor4(gf_mul_table<1, true>(left, tb, 0), v);
            }
            v = make_uint4(__shfl_sync(0xffffffffu, v.x, 31), __shfl_sync(0xffffffffu, v.y, 31),
                           __shfl_sync(0xffffffffu, v.z, 31), __shfl_sync(0xffffffffu, v.w, 31));
            acc = k0 == 0 ? v : xor4(gf_mul_warp<true>(acc, L.h.join_pow + 4 * 512, lane), v);
            k0 += cnt;
        }
        finish_record(r, xor4(acc, mask), tag_in);
    }
}

// ----------------------------------------------------------------------------
// Writeback quantisation (transport_codec.py:22-42), one thread per group.
// ----------------------------------------------------------------------------
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }

// q = clamp(round_half_even(fl((x - low) / scale)), 0, levels) without a
// division per element: y = fl(fl(x - low) * fl(1 / scale)) differs from the
// correctly rounded quotient Q by at most Q * 1.8e-7 <= 4.7e-5 (Q <= 256:
// two roundings of 2^-24 relative error each, on top of Q's own rounding), so
// round(y) == round(Q) unless y lies within 2^-13 of a half-integer; a row
// holding such an element (or an exact tie) is redone with IEEE divisions.
//
// Rounding uses the fp32 adder: for 0 <= y < 2^22, m = fl(y + 1.5 * 2^23) holds
// round_half_even(y) in its low mantissa bits, so neither a rounding nor a
// conversion instruction is needed (y >= 0 because low is the group minimum).
constexpr float kRoundMagic = 12582912.0f;   // 1.5 * 2^23

// Quantises the 8 elements of one row slice into m[c] = fl(y + magic), whose
// low byte is q = round(y) (q <= 255, and y <= levels (1 + 2^-23), so no
// clamp is needed).  |y - round(y)| is exact; elements within 2^-13 of a
// half-integer are flagged in the returned mask for the exact division.
template <class Val, class Low, class Inv>
__device__ __forceinline__ uint32_t quantise8_fast(Val val, Low low, Inv inv, uint32_t (&m)[8])
{
    uint32_t near = 0;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const float y = __fmul_rn(__fsub_rn(val(c), low(c)), inv(c));
        const float mf = __fadd_rn(y, kRoundMagic);
        if (fabsf(__fsub_rn(y, __fsub_rn(mf, kRoundMagic))) > 0.5f - 0x1p-13f) near |= 1u << c;
        m[c] = __float_as_uint(mf);
    }
    return near;
}

// The reference's division for one element (rare path).
__device__ __noinline__ uint32_t quantise_exact(float x, float low, float scale)
{
    return __float_as_uint(__fadd_rn(__fdiv_rn(__fsub_rn(x, low), scale), kRoundMagic));
}

// Packs m[0..7] (q in the low byte) as 8 int8 bytes or 8 int4 nibbles (even
// element in the low nibble).
template <int BITS>
__device__ __forceinline__ uint2 pack8(const uint32_t (&m)[8])
{
    if (BITS == 8) {
        const uint32_t w0 = __byte_perm(__byte_perm(m[0], m[1], 0x0040u), __byte_perm(m[2], m[3], 0x0040u), 0x5410u);
        const uint32_t w1 = __byte_perm(__byte_perm(m[4], m[5], 0x0040u), __byte_perm(m[6], m[7], 0x0040u), 0x5410u);
        return make_uint2(w0, w1);
    }
    // Low byte of m[c] + (m[c+1] << 4) is q[c] + 16 q[c+1] (both <= 15).
    const uint32_t t0 = m[0] + (m[1] << 4), t1 = m[2] + (m[3] << 4);
    const uint32_t t2 = m[4] + (m[5] << 4), t3 = m[6] + (m[7] << 4);
    return make_uint2(__byte_perm(__byte_perm(t0, t1, 0x0040u), __byte_perm(t2, t3, 0x0040u), 0x5410u), 0u);
}

// Tiled quantisation: one CTA of 256 threads per (record, 64-token group,
// CW-channel chunk).  Thread (row slot, lane-in-row) loads 16 bytes (8
// channels) of each of its rows with coalesced 16-byte loads and keeps them
// (packed bf16) in registers.  K groups (64 tokens of one channel) reduce
// over the thread's rows and the row slots (shared memory, laid out so both
// the partial writes and the final reads are conflict-free); V groups (64
// dims of one token/head) reduce over the 8 lanes that hold the group.
// Quantised bytes go out as 8-byte (int8) or 4-byte (int4) coalesced stores,
// element e = token * hd + channel.  Three CTAs per SM (80 registers, a
// small spill in the 256-channel variant) keep more loads in flight than two:
// measured 24.6 against 26.5 us per c4 layer.
template <int CW, int BITS>
__global__ void __launch_bounds__(256, 3) kv_encode_kernel(const __grid_constant__ EncodeLaunch L)
{
    constexpr int kTpr = CW / 8;                 // threads per row
    constexpr int kRowsPerPass = 256 / kTpr;
    constexpr int kPasses = 64 / kRowsPerPass;
    constexpr uint32_t kLevels = (1u << BITS) - 1u;
    __shared__ float red_lo[kRowsPerPass][8][kTpr], red_hi[kRowsPerPass][8][kTpr];
    __shared__ float fin_lo[8][kTpr], fin_sc[8][kTpr], fin_inv[8][kTpr];

    const CodecParams cp = L.codec;
    const uint32_t hd = cp.heads * 128u;
    const uint32_t chunks = hd / CW;
    const uint32_t rec = blockIdx.y;
    const uint32_t tg = blockIdx.x / chunks, chunk = blockIdx.x % chunks;
    const uint32_t kind = rec >= L.v_first ? 1u : 0u;
    const uint32_t tid = threadIdx.x, slot = tid / kTpr, tl = tid % kTpr;
    const uint32_t c0 = chunk * CW + 8u * tl;                 // first of the thread's 8 channels
    const uint8_t* src = static_cast<const uint8_t*>(L.srcs[rec]);
    uint8_t* pkt = L.packets + static_cast<size_t>(rec) * L.width;
    float* scale = reinterpret_cast<float*>(pkt + cp.qb);
    float* lowp = reinterpret_cast<float*>(pkt + cp.qb + cp.sb);
    const float levels = static_cast<float>(kLevels);

    uint4 raw[kPasses];
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
        const uint32_t t = tg * 64u + p * kRowsPerPass + slot;
        raw[p] = __ldg(reinterpret_cast<const uint4*>(src + (static_cast<size_t>(t) * hd + c0) * 2u));
    }
    auto val = [&](int p, int c) {
        const uint32_t w = c < 2 ? raw[p].x : c < 4 ? raw[p].y : c < 6 ? raw[p].z : raw[p].w;
        return bf16_bits_to_f32((c & 1) ? (w >> 16) : (w & 0xffffu));
    };

    float lo[8], sc[8], inv[8];   // K: per channel of the thread; V: per pass (group of the row)
    if (kind == 0) {
        // Per-channel min/max over the thread's rows on packed bf16 pairs
        // (exact: min and max select one of the inputs).
        __nv_bfloat162 l2[4], h2[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const uint32_t first = w == 0 ? raw[0].x : w == 1 ? raw[0].y : w == 2 ? raw[0].z : raw[0].w;
            l2[w] = h2[w] = *reinterpret_cast<const __nv_bfloat162*>(&first);
#pragma unroll
            for (int p = 1; p < kPasses; ++p) {
                const uint32_t v = w == 0 ? raw[p].x : w == 1 ? raw[p].y : w == 2 ? raw[p].z : raw[p].w;
                const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&v);
                l2[w] = __hmin2(l2[w], b);
                h2[w] = __hmax2(h2[w], b);
            }
        }
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            red_lo[slot][2 * w][tl] = __low2float(l2[w]);
            red_lo[slot][2 * w + 1][tl] = __high2float(l2[w]);
            red_hi[slot][2 * w][tl] = __low2float(h2[w]);
            red_hi[slot][2 * w + 1][tl] = __high2float(h2[w]);
        }
        __syncthreads();
        if (tid < CW) {
            // channel chunk * CW + 8 * ttl + cc
            const uint32_t ttl = tid % kTpr, cc = tid / kTpr;
            float l = red_lo[0][cc][ttl], h = red_hi[0][cc][ttl];
#pragma unroll
            for (int r = 1; r < kRowsPerPass; ++r) {
                l = fminf(l, red_lo[r][cc][ttl]);
                h = fmaxf(h, red_hi[r][cc][ttl]);
            }
            const float s1 = fmaxf(__fdiv_rn(__fsub_rn(h, l), levels), 1e-12f);
            fin_lo[cc][ttl] = l;
            fin_sc[cc][ttl] = s1;
            fin_inv[cc][ttl] = __frcp_rn(s1);
            const uint32_t sidx = tg * hd + chunk * CW + 8u * ttl + cc;
            scale[sidx] = s1;
            lowp[sidx] = l;
        }
        __syncthreads();
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            lo[c] = fin_lo[c][tl];
            sc[c] = fin_sc[c][tl];
            inv[c] = fin_inv[c][tl];
        }
    } else {
        // V: the 8 lanes of a 64-dim group reduce each pass's group; lane j of
        // the group then divides for pass j, and the passes fetch their scale
        // and reciprocal from that lane.
        float vl[kPasses], vh[kPasses];
#pragma unroll
        for (int p = 0; p < kPasses; ++p) {
            const __nv_bfloat162 w0 = *reinterpret_cast<const __nv_bfloat162*>(&raw[p].x);
            const __nv_bfloat162 w1 = *reinterpret_cast<const __nv_bfloat162*>(&raw[p].y);
            const __nv_bfloat162 w2 = *reinterpret_cast<const __nv_bfloat162*>(&raw[p].z);
            const __nv_bfloat162 w3 = *reinterpret_cast<const __nv_bfloat162*>(&raw[p].w);
            const __nv_bfloat162 l2 = __hmin2(__hmin2(w0, w1), __hmin2(w2, w3));
            const __nv_bfloat162 h2 = __hmax2(__hmax2(w0, w1), __hmax2(w2, w3));
            float l = fminf(__low2float(l2), __high2float(l2)), h = fmaxf(__low2float(h2), __high2float(h2));
#pragma unroll
            for (int m = 1; m < 8; m <<= 1) {
                l = fminf(l, __shfl_xor_sync(0xffffffffu, l, m));
                h = fmaxf(h, __shfl_xor_sync(0xffffffffu, h, m));
            }
            vl[p] = l;
            vh[p] = h;
        }
        const uint32_t j = tl & 7u;
        float lj = vl[0], hj = vh[0];
#pragma unroll
        for (int p = 1; p < kPasses; ++p)
            if (j == static_cast<uint32_t>(p)) { lj = vl[p]; hj = vh[p]; }
        const float sj = fmaxf(__fdiv_rn(__fsub_rn(hj, lj), levels), 1e-12f);
        const float ij = __frcp_rn(sj);
        if (j < static_cast<uint32_t>(kPasses)) {
            const uint32_t t = tg * 64u + j * kRowsPerPass + slot;
            const uint32_t sidx = (t * hd + c0 - 8u * j) / 64u;   // group start channel = c0 - 8 j
            scale[sidx] = sj;
            lowp[sidx] = lj;
        }
        const uint32_t base_lane = (tid & 31u) & ~7u;
#pragma unroll
        for (int p = 0; p < kPasses; ++p) {
            const float sp = __shfl_sync(0xffffffffu, sj, base_lane | p);
            const float ip = __shfl_sync(0xffffffffu, ij, base_lane | p);
            // stash per pass in the K arrays' slots (8 >= kPasses)
            lo[p] = vl[p];
            sc[p] = sp;
            inv[p] = ip;
        }
    }
    // One row slice: quantise, redo flagged elements exactly, pack, store.
    auto row = [&](int p, auto low, auto scl, auto inv_of) {
        const uint32_t t = tg * 64u + p * kRowsPerPass + slot;
        uint32_t m[8];
        const uint32_t near = quantise8_fast([&](int c) { return val(p, c); }, low, inv_of, m);
        if (near) {
#pragma unroll
            for (int c = 0; c < 8; ++c)
                if (near & (1u << c)) m[c] = quantise_exact(val(p, c), low(c), scl(c));
        }
        const uint2 word = pack8<BITS>(m);
        const size_t e0 = static_cast<size_t>(t) * hd + c0;
        if (BITS == 8)
            *reinterpret_cast<uint2*>(pkt + e0) = word;
        else
            *reinterpret_cast<uint32_t*>(pkt + e0 / 2) = word.x;
    };
    if (kind == 0) {
#pragma unroll
        for (int p = 0; p < kPasses; ++p)
            row(p, [&](int c) { return lo[c]; }, [&](int c) { return sc[c]; }, [&](int c) { return inv[c]; });
    } else {
#pragma unroll
        for (int p = 0; p < kPasses; ++p)
            row(p, [&](int) { return lo[p]; }, [&](int) { return sc[p]; }, [&](int) { return inv[p]; });
    }
    if (blockIdx.x == 0) {
        // int32 header {1, layer, kind, bits} then zero padding to width.
        const uint32_t hdr = cp.qb + 2u * cp.sb;
        for (uint32_t i = tid; i < L.width - hdr; i += blockDim.x) {
            uint8_t b = 0;
            if (i < 16) {
                const uint32_t word = i < 4 ? 1u : i < 8 ? L.layer : i < 12 ? kind : cp.bits;
                b = static_cast<uint8_t>(word >> (8 * (i & 3)));
            }
            pkt[hdr + i] = b;
        }
    }
}

// Device side of the session key agreement (key_agreement.aicpu): a device
// X25519 key pair, the shared secret with the host's public value, the
// session key and the proof the host checks.  B200 has no entropy source, so
// the device secret is a BLAKE2b-512 hash of %globaltimer and clock64 readings
// that 32 threads take around contended shared-memory atomics: far weaker
// than the AICPU's /dev/urandom, so callers that can supply a host-agreed key
// (secure_infer_session_init) should.
__global__ void __launch_bounds__(32) key_agreement_kernel(const uint8_t* host_public, const uint8_t* challenge,
                                                           uint8_t* device_key, uint8_t* device_public,
                                                           uint8_t* proof, int32_t* status)
{
    __shared__ unsigned long long samples[32][8];
    __shared__ uint32_t contended;
    const uint32_t lane = threadIdx.x;
    if (lane == 0) {
        contended = 0;
        *status = 1;
    }
    __syncwarp();
    for (int i = 0; i < 8; ++i) {
        const uint32_t spins = 64u + (lane * 7u + static_cast<uint32_t>(i)) % 13u;
        for (uint32_t j = 0; j < spins; ++j) atomicAdd(&contended, lane ^ j);
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        samples[lane][i] = t ^ (static_cast<unsigned long long>(clock64()) << 17) ^ contended;
    }
    __syncwarp();
    if (lane != 0) return;
    uint8_t secret[64], shared[32];
    kx::blake2b(secret, 64, nullptr, 0, reinterpret_cast<const uint8_t*>(samples), sizeof(samples));
    *status = 2;
    kx::x25519_public(device_public, secret);
    kx::x25519(shared, secret, host_public);
    uint32_t nonzero = 0;
    for (int i = 0; i < 32; ++i) nonzero |= shared[i];
    if (nonzero) {
        *status = 3;
        kx::derive_key(device_key, shared, host_public, device_public, challenge);
        kx::derive_proof(proof, device_key, challenge);
        *status = 0;
    }
    for (int i = 0; i < 64; ++i) secret[i] = 0;
    for (int i = 0; i < 32; ++i) shared[i] = 0;
}

int launch_key_agreement(const void* host_public, const void* challenge, void* device_key, void* device_public,
                         void* proof, int32_t* status, cudaStream_t stream)
{
    key_agreement_kernel<<<1, 32, 0, stream>>>(static_cast<const uint8_t*>(host_public),
                                               static_cast<const uint8_t*>(challenge),
                                               static_cast<uint8_t*>(device_key),
                                               static_cast<uint8_t*>(device_public), static_cast<uint8_t*>(proof),
                                               status);
    return cudaGetLastError();
}

__global__ void auth_gate_kernel(uint8_t* data, const uint32_t* status, uint64_t bytes)
{
    if (__ldg(status) == 1u) return;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < bytes;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
        data[i] = 0;
}

// ----------------------------------------------------------------------------
// Host launchers
// ----------------------------------------------------------------------------
namespace {

struct DeviceInfo {
    int sms = 0;
    bool ctr_attr_set = false;
    int seg_blocks_per_sm[4] = {0, 0, 0, 0};
    bool attr_set[4] = {false, false, false, false};
};

std::mutex g_dev_mu;
DeviceInfo g_dev[64];

DeviceInfo& device_info(int dev)
{
    DeviceInfo& d = g_dev[dev & 63];
    if (d.sms == 0) cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    return d;
}

// SMs a layer launch may occupy (0: all).  A caller that alternates
// consecutive layers between streams sets it to a share of the GPU so the
// launches of different streams run side by side instead of queueing for the
// same SMs.
std::atomic<uint32_t> g_layer_sm_limit{0};

int layer_sms(const DeviceInfo& d)
{
    const uint32_t lim = g_layer_sm_limit.load(std::memory_order_relaxed);
    return lim != 0 && static_cast<int>(lim) < d.sms ? static_cast<int>(lim) : d.sms;
}

// ---------------------------------------------------------------- profile
struct ProfileRec {
    uint32_t kind;
    cudaEvent_t start, end;
};
std::atomic<bool> g_prof_on{false};
std::mutex g_prof_mu;
std::vector<ProfileRec> g_prof_recs;
std::vector<cudaEvent_t> g_prof_pool;

cudaEvent_t prof_event()
{
    if (!g_prof_pool.empty()) {
        cudaEvent_t e = g_prof_pool.back();
        g_prof_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

// Brackets one launch with timing events when profiling is on.
class ProfileScope {
public:
    ProfileScope(uint32_t kind, cudaStream_t stream) : stream_(stream)
    {
        if (!g_prof_on.load(std::memory_order_relaxed)) return;
        std::lock_guard<std::mutex> lock(g_prof_mu);
        rec_ = ProfileRec{kind, prof_event(), prof_event()};
        active_ = rec_.start && rec_.end && cudaEventRecord(rec_.start, stream) == cudaSuccess;
    }
    ~ProfileScope()
    {
        if (!active_) return;
        std::lock_guard<std::mutex> lock(g_prof_mu);
        cudaEventRecord(rec_.end, stream_);
        g_prof_recs.push_back(rec_);
    }

private:
    cudaStream_t stream_;
    ProfileRec rec_{};
    bool active_ = false;
};

template <bool A>
int segment_launch_impl(const SegmentLaunch& args, size_t smem, int variant, cudaStream_t stream)
{
    int dev = 0;
    cudaGetDevice(&dev);
    int per_sm = 0, sms = 0;
    {
        std::lock_guard<std::mutex> lock(g_dev_mu);
        DeviceInfo& d = device_info(dev);
        if (!d.attr_set[variant]) {
            const size_t max_smem = kGhashSmem + kAesSmem;
            cudaError_t e = cudaFuncSetAttribute(gcm_segment_kernel<A>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(max_smem));
            if (e != cudaSuccess) return e;
            e = cudaFuncSetAttribute(gcm_segment_kernel<A>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     cudaSharedmemCarveoutMaxShared);
            if (e != cudaSuccess) return e;
            d.attr_set[variant] = true;
        }
        sms = d.sms;
        per_sm = d.seg_blocks_per_sm[variant];
    }
    if (per_sm == 0) {
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gcm_segment_kernel<A>, kThreads, smem);
        if (per_sm < 1) per_sm = 1;
        std::lock_guard<std::mutex> lock(g_dev_mu);
        device_info(dev).seg_blocks_per_sm[variant] = per_sm;
    }
    const uint32_t grid = static_cast<uint32_t>(
        args.total_segs < static_cast<uint32_t>(sms * per_sm) ? args.total_segs : sms * per_sm);
    ProfileScope prof(kKernSegment, stream);
    gcm_segment_kernel<A><<<grid, kThreads, smem, stream>>>(args);
    return cudaGetLastError();
}

}  // namespace

uint32_t set_layer_sm_limit(uint32_t sms) { return g_layer_sm_limit.exchange(sms); }

void profile_enable(bool on) { g_prof_on.store(on); }

int profile_collect(double* total_us, uint64_t* launches, uint32_t kinds)
{
    std::lock_guard<std::mutex> lock(g_prof_mu);
    for (uint32_t k = 0; k < kinds; ++k) {
        if (total_us) total_us[k] = 0.0;
        if (launches) launches[k] = 0;
    }
    int rc = 0;
    for (const ProfileRec& r : g_prof_recs) {
        float ms = 0.0f;
        if (cudaEventSynchronize(r.end) != cudaSuccess || cudaEventElapsedTime(&ms, r.start, r.end) != cudaSuccess)
            rc = -1;
        else if (r.kind < kinds) {
            if (total_us) total_us[r.kind] += 1e3 * ms;
            if (launches) ++launches[r.kind];
        }
        g_prof_pool.push_back(r.start);
        g_prof_pool.push_back(r.end);
    }
    g_prof_recs.clear();
    return rc;
}

const char* kernel_kind_name(uint32_t kind)
{
    static const char* names[kKernKinds] = {"gcm_layer_ctr_kernel", "gcm_layer_verify_kernel", "gcm_layer_encrypt",
                                            "kv_encode_kernel", "gcm_segment_kernel", "gcm_ctr_kernel",
                                            "gcm_schedule_kernel", "auth_gate_kernel",
                                            "gcm_layer_verify_inline_kernel", "gcm_layer_ctr_bs_kernel"};
    return kind < kKernKinds ? names[kind] : nullptr;
}

size_t schedule_bytes() { return sizeof(GcmSchedule); }

uint32_t segments_for(uint64_t count, uint32_t aad_bytes, uint32_t seg_blocks)
{
    const uint64_t m = (aad_bytes + 15u) / 16u + (count + 15u) / 16u + 1u;
    const uint64_t n = m / (seg_blocks ? seg_blocks : kSegBlocks);
    return static_cast<uint32_t>(n ? n : 1u);
}

uint32_t segment_blocks_for(uint64_t total_blocks)
{
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    {
        std::lock_guard<std::mutex> lock(g_dev_mu);
        sms = device_info(dev).sms;
    }
    uint32_t sb = kSegBlocks;
    while (sb > 256u && total_blocks / sb < 2u * static_cast<uint64_t>(sms)) sb >>= 1;
    return sb;
}

int launch_join_tables(const GcmSchedule* sched, void* out, cudaStream_t stream)
{
    gcm_join_tables_kernel<<<kMaxWarpSegSteps, 32, 0, stream>>>(sched, static_cast<uint4*>(out));
    return cudaGetLastError();
}

int launch_schedule(GcmSchedule* sched, const void* key, const void* h, bool need_tables, cudaStream_t stream)
{
    ProfileScope prof(kKernSchedule, stream);
    gcm_schedule_kernel<<<1, 256, 0, stream>>>(static_cast<const uint8_t*>(key), static_cast<const uint8_t*>(h),
                                               sched, need_tables ? 1 : 0);
    return cudaGetLastError();
}

int launch_ctr(const CtrLaunch& args, cudaStream_t stream)
{
    if (args.total_blocks == 0) return cudaSuccess;
    const CtrJob* jobs = args.jobs ? nullptr : args.inl;
    uint64_t uniform = 0;
    if (jobs) {
        const uint64_t b0 = (jobs[0].bytes + 15) / 16;
        bool same = true;
        for (uint32_t i = 0; i < args.njobs; ++i) same = same && (jobs[i].bytes + 15) / 16 == b0 && jobs[i].block_first == i * b0;
        uniform = same ? b0 : 0;
    }
    return launch_ctr_uniform(args, uniform, stream);
}

int launch_ctr_uniform(const CtrLaunch& args, uint64_t uniform_blocks, cudaStream_t stream)
{
    if (args.total_blocks == 0) return cudaSuccess;
    int dev = 0;
    cudaGetDevice(&dev);
    int sms;
    {
        std::lock_guard<std::mutex> lock(g_dev_mu);
        DeviceInfo& d = device_info(dev);
        sms = d.sms;
        if (!d.ctr_attr_set) {
            cudaError_t e = cudaFuncSetAttribute(gcm_ctr_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(kCtrSmem));
            if (e != cudaSuccess) return e;
            e = cudaFuncSetAttribute(gcm_ctr_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     cudaSharedmemCarveoutMaxShared);
            if (e != cudaSuccess) return e;
            d.ctr_attr_set = true;
        }
    }
    const uint64_t want = (args.total_blocks + kCtrThreads - 1) / kCtrThreads;
    const uint64_t cap = static_cast<uint64_t>(sms);
    const uint32_t grid = static_cast<uint32_t>(want < cap ? want : cap);
    ProfileScope prof(kKernCtr, stream);
    gcm_ctr_kernel<<<grid, kCtrThreads, kCtrSmem, stream>>>(args, uniform_blocks);
    return cudaGetLastError();
}

void layer_segments_for(uint64_t count, uint32_t n, uint32_t codec_bits, uint32_t* seg_steps, uint32_t* nseg)
{
    // Pick the segment length (32 k blocks, k <= 64) so that n * nseg fills
    // the resident warps once (one CTA per SM); long layers fall back to the
    // longest segment.
    const uint32_t kLayerWarps = layer_threads(codec_bits ? kLayerVerifyCodec8 : kLayerVerifyRaw) / 32;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    {
        std::lock_guard<std::mutex> lock(g_dev_mu);
        sms = layer_sms(device_info(dev));
    }
    const uint64_t m = 4u + (count + 15u) / 16u + 1u;
    const uint64_t warps = static_cast<uint64_t>(sms) * kLayerWarps;
    const uint64_t per_record = warps / (n ? n : 1u);
    uint64_t k = per_record ? (m + 32u * per_record - 1) / (32u * per_record) : kMaxWarpSegSteps;
    if (k < 1) k = 1;
    if (k > static_cast<uint64_t>(kMaxWarpSegSteps)) k = kMaxWarpSegSteps;
    *seg_steps = static_cast<uint32_t>(k);
    *nseg = static_cast<uint32_t>((m + 32u * k - 1) / (32u * k));
}

template <int kCap, class Kernel>
int layer_launch(uint32_t kind, Kernel kernel, const LayerHeader& h, const LayerRec* rec, uint32_t threads,
                 size_t smem, uint32_t items, bool& attr_set, cudaStream_t stream, uint32_t ctas_per_sm = 1)
{
    int dev = 0;
    cudaGetDevice(&dev);
    int sms;
    {
        std::lock_guard<std::mutex> lock(g_dev_mu);
        sms = layer_sms(device_info(dev));
        if (!attr_set) {
            cudaError_t e =
                cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
            if (e != cudaSuccess) return e;
            // Same (maximum) shared-memory carve-out for every large-table
            // kernel, so back-to-back launches never reconfigure L1.
            e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     cudaSharedmemCarveoutMaxShared);
            if (e != cudaSuccess) return e;
            attr_set = true;
        }
    }
    LayerLaunch<kCap> L;
    L.h = h;
    for (uint32_t i = 0; i < h.n; ++i) L.rec[i] = rec[i];
    const uint32_t cap = static_cast<uint32_t>(sms) * ctas_per_sm;
    const uint32_t grid = items < cap ? items : cap;
    // Programmatic stream serialisation: the kernel's launch and table
    // prologue overlap the tail of the previous layer kernel in the stream.
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ProfileScope prof(kind, stream);
    return cudaLaunchKernelEx(&cfg, kernel, L);
}

// SECURE_INFER_AES_KEYSTREAM=bitsliced selects the bitsliced keystream kernel
// (read at every launch); the T-table kernel is the default.
bool keystream_bitsliced()
{
    const char* v = std::getenv("SECURE_INFER_AES_KEYSTREAM");
    return v != nullptr && v[0] == 'b';
}

int launch_layer_keystream(const LayerHeader& h, const LayerRec* rec, cudaStream_t stream)
{
    if (h.n == 0) return cudaSuccess;
    if (h.n > static_cast<uint32_t>(kLayerCapLarge)) return cudaErrorInvalidValue;
    if (keystream_bitsliced()) {
        static bool bs_small[64], bs_large[64];
        int dev = 0;
        cudaGetDevice(&dev);
        const uint32_t groups = static_cast<uint32_t>(((h.count + 15) / 16 + 2 + 31) / 32);
        const uint32_t items = (groups * h.n + kBsThreads - 1) / kBsThreads;
        if (h.n <= static_cast<uint32_t>(kLayerCapSmall))
            return layer_launch<kLayerCapSmall>(kKernLayerCtrBitsliced, gcm_layer_ctr_bs_kernel<kLayerCapSmall>, h, rec,
                                                kBsThreads, 0, items, bs_small[dev & 63], stream);
        return layer_launch<kLayerCapLarge>(kKernLayerCtrBitsliced, gcm_layer_ctr_bs_kernel<kLayerCapLarge>, h, rec,
                                            kBsThreads, 0, items, bs_large[dev & 63], stream);
    }
    const uint32_t blocks = static_cast<uint32_t>(((h.count + 15) / 16 + 1) * h.n);
    const uint32_t items = (blocks + kLayerCtrThreads - 1) / kLayerCtrThreads;
    static bool set_small[64], set_large[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (h.n <= static_cast<uint32_t>(kLayerCapSmall))
        return layer_launch<kLayerCapSmall>(kKernLayerCtr, gcm_layer_ctr_kernel<kLayerCapSmall>, h, rec, kLayerCtrThreads, kCtrSmem, items,
                                            set_small[dev & 63], stream);
    return layer_launch<kLayerCapLarge>(kKernLayerCtr, gcm_layer_ctr_kernel<kLayerCapLarge>, h, rec, kLayerCtrThreads, kCtrSmem, items,
                                        set_large[dev & 63], stream);
}

int launch_layer_verify(const LayerHeader& h, const LayerRec* rec, cudaStream_t stream)
{
    if (h.n == 0) return cudaSuccess;
    if (h.n > static_cast<uint32_t>(kLayerCapLarge) || h.join_pow == nullptr || h.seg_steps < 1 ||
        h.seg_steps > static_cast<uint32_t>(kMaxWarpSegSteps))
        return cudaErrorInvalidValue;
    const uint32_t items = h.nseg * h.n;
    static bool set_small[64], set_large[64];
    int dev = 0;
    cudaGetDevice(&dev);
    // One CTA per SM (160 KiB of tables in shared memory).
    static bool set_small_8[64], set_large_8[64], set_small_4[64], set_large_4[64];
    const uint32_t warps = layer_threads(h.codec.bits ? kLayerVerifyCodec8 : kLayerVerifyRaw) / 32;
    const uint32_t grid = (items + warps - 1) / warps;
    const bool small = h.n <= static_cast<uint32_t>(kLayerCapSmall);
    if (h.codec.bits == 8) {
        if (small)
            return layer_launch<kLayerCapSmall>(kKernLayerVerify, gcm_layer_verify_kernel<kLayerCapSmall, kLayerVerifyCodec8>,
                                                h, rec, layer_threads(kLayerVerifyCodec8), kLayerSmem, grid, set_small_8[dev & 63], stream, 1);
        return layer_launch<kLayerCapLarge>(kKernLayerVerify, gcm_layer_verify_kernel<kLayerCapLarge, kLayerVerifyCodec8>,
                                            h, rec, layer_threads(kLayerVerifyCodec8), kLayerSmem, grid, set_large_8[dev & 63], stream, 1);
    }
    if (h.codec.bits == 4) {
        if (small)
            return layer_launch<kLayerCapSmall>(kKernLayerVerify, gcm_layer_verify_kernel<kLayerCapSmall, kLayerVerifyCodec4>,
                                                h, rec, layer_threads(kLayerVerifyCodec4), kLayerSmem, grid, set_small_4[dev & 63], stream, 1);
        return layer_launch<kLayerCapLarge>(kKernLayerVerify, gcm_layer_verify_kernel<kLayerCapLarge, kLayerVerifyCodec4>,
                                            h, rec, layer_threads(kLayerVerifyCodec4), kLayerSmem, grid, set_large_4[dev & 63], stream, 1);
    }
    if (small)
        return layer_launch<kLayerCapSmall>(kKernLayerVerify, gcm_layer_verify_kernel<kLayerCapSmall, kLayerVerifyRaw>, h, rec,
                                            layer_threads(kLayerVerifyRaw), kLayerSmem, grid, set_small[dev & 63], stream, 1);
    return layer_launch<kLayerCapLarge>(kKernLayerVerify, gcm_layer_verify_kernel<kLayerCapLarge, kLayerVerifyRaw>, h, rec,
                                        layer_threads(kLayerVerifyRaw), kLayerSmem, grid, set_large[dev & 63], stream, 1);
}

int launch_layer_verify_inline(const LayerHeader& h, const LayerRec* rec, cudaStream_t stream)
{
    if (h.n == 0) return cudaSuccess;
    if (h.n > static_cast<uint32_t>(kLayerCapLarge) || h.join_pow == nullptr || h.seg_steps < 1 ||
        h.seg_steps > static_cast<uint32_t>(kMaxWarpSegSteps) || h.unaligned || h.codec.bits)
        return cudaErrorInvalidValue;
    static bool set_small[64], set_large[64];
    int dev = 0;
    cudaGetDevice(&dev);
    const uint32_t warps = kInlineThreads / 32;
    const uint32_t grid = (h.nseg * h.n + warps - 1) / warps;
    if (h.n <= static_cast<uint32_t>(kLayerCapSmall))
        return layer_launch<kLayerCapSmall>(kKernLayerVerifyInline, gcm_layer_verify_inline_kernel<kLayerCapSmall>, h,
                                            rec, kInlineThreads, kInlineSmem, grid, set_small[dev & 63], stream, 1);
    return layer_launch<kLayerCapLarge>(kKernLayerVerifyInline, gcm_layer_verify_inline_kernel<kLayerCapLarge>, h, rec,
                                        kInlineThreads, kInlineSmem, grid, set_large[dev & 63], stream, 1);
}

int launch_layer_encrypt(const LayerHeader& h, const LayerRec* rec, cudaStream_t stream)
{
    if (h.n == 0) return cudaSuccess;
    if (h.n > static_cast<uint32_t>(kLayerCapLarge) || h.aad == nullptr || h.join_pow == nullptr ||
        h.seg_steps < 1 || h.seg_steps > static_cast<uint32_t>(kMaxWarpSegSteps))
        return cudaErrorInvalidValue;
    const uint32_t items = h.nseg * h.n;
    static bool set_small[64], set_large[64];
    int dev = 0;
    cudaGetDevice(&dev);
    const uint32_t warps = layer_threads(kLayerEncrypt) / 32;
    const uint32_t grid = (items + warps - 1) / warps;
    if (h.n <= static_cast<uint32_t>(kLayerCapSmall))
        return layer_launch<kLayerCapSmall>(kKernLayerEncrypt, gcm_layer_verify_kernel<kLayerCapSmall, kLayerEncrypt>, h, rec,
                                            layer_threads(kLayerEncrypt), kLayerSmem, grid, set_small[dev & 63], stream, 1);
    return layer_launch<kLayerCapLarge>(kKernLayerEncrypt, gcm_layer_verify_kernel<kLayerCapLarge, kLayerEncrypt>, h, rec,
                                        layer_threads(kLayerEncrypt), kLayerSmem, grid, set_large[dev & 63], stream, 1);
}

int launch_segments(const SegmentLaunch& args, bool inline_aes, cudaStream_t stream)
{
    if (args.total_segs == 0) return cudaSuccess;
    const size_t smem = kGhashSmem + (inline_aes ? kAesSmem : 0);
    if (inline_aes) return segment_launch_impl<true>(args, smem, 1, stream);
    return segment_launch_impl<false>(args, smem, 0, stream);
}

int launch_encode(const EncodeLaunch& args, cudaStream_t stream)
{
    if (args.n == 0) return cudaSuccess;
    const uint32_t hd = args.codec.heads * 128u;
    const bool wide = hd % 256u == 0;
    const dim3 grid(2u * (hd / (wide ? 256u : 128u)), args.n);
    ProfileScope prof(kKernEncode, stream);
    if (args.codec.bits == 8) {
        if (wide) kv_encode_kernel<256, 8><<<grid, 256, 0, stream>>>(args);
        else kv_encode_kernel<128, 8><<<grid, 256, 0, stream>>>(args);
    } else {
        if (wide) kv_encode_kernel<256, 4><<<grid, 256, 0, stream>>>(args);
        else kv_encode_kernel<128, 4><<<grid, 256, 0, stream>>>(args);
    }
    return cudaGetLastError();
}

int launch_auth_gate(uint8_t* data, const uint32_t* status, uint64_t bytes, cudaStream_t stream)
{
    const uint64_t want = (bytes + 255) / 256;
    const uint32_t grid = static_cast<uint32_t>(want < 1024 ? (want ? want : 1) : 1024);
    ProfileScope prof(kKernAuthGate, stream);
    auth_gate_kernel<<<grid, 256, 0, stream>>>(data, status, bytes);
    return cudaGetLastError();
}

}  // namespace sib

// ----------------------------------------------------------------------------
// Allocation-free entry point.
// ----------------------------------------------------------------------------
// Some callers cannot call cudaMalloc: code running under an allocator or
// memory budget they do not own, or paths that must never pay for a first-call
// device allocation.  The plugin entry points above allocate one scratch area
// per stream on first use.  secure_infer_aicpu_gcm_decrypt_verify_aad_noalloc_do
// runs the same key-schedule and fused decrypt/verify kernels with their
// scratch in the fixed array below instead, so it never allocates.
#include <cstdio>

namespace sib {
namespace {

constexpr uint64_t kNoAllocMaxBytes = 16ull << 20;   // payload bytes per call
constexpr uint64_t kNoAllocMaxAad = 4096;             // AAD bytes per call
constexpr uint32_t kNoAllocMaxSegs =
    static_cast<uint32_t>((kNoAllocMaxAad / 16 + kNoAllocMaxBytes / 16 + 1) / kSegBlocks + 1);

struct NoAllocScratch {
    GcmSchedule sched;                 // key schedule (rebuilt when key or H change)
    uint4 partials[kNoAllocMaxSegs];   // per-segment GHASH partials
    uint32_t counters[4];              // segment arrival counter (must start at zero)
};

}  // namespace
}  // namespace sib

// The scratch itself: about 1 MiB, held by every GPU that loads this library
// until the process exits.  Static device memory starts zeroed.
static __device__ __align__(256) uint8_t g_noalloc_scratch[sizeof(sib::NoAllocScratch)];

namespace sib {
namespace {

// Device address of g_noalloc_scratch on the current device.  In host code the
// array's name is only a host-side stand-in; the address comes from the
// runtime with the device current.  It is looked up on every call rather than
// cached: after cudaDeviceReset the module is loaded again and the array may
// move, and the lookup costs a few microseconds of host time.
NoAllocScratch* noalloc_scratch()
{
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return nullptr;
    return static_cast<NoAllocScratch*>(p);
}

}  // namespace
}  // namespace sib

// Same arguments, meaning and results as
// secure_infer_aicpu_gcm_decrypt_verify_aad_do; returns -2 (with a message on
// stderr) when bytes exceed 16 MiB or aad_bytes exceed 4096.  Every call looks
// up the scratch address of the current device; the first call on a device may
// load the module, so make it before any stream capture.
// All calls share the one scratch array: calls whose work overlaps on the GPU
// (for example on two streams at once) race and must be serialised by the
// caller.
extern "C" __attribute__((visibility("default"))) int secure_infer_aicpu_gcm_decrypt_verify_aad_noalloc_do(
    void* stream, void* ciphertext, void* key, void* hash_subkey, void* expected_tag, void* plaintext_output,
    void* status_output, uint64_t bytes, uint32_t iv_word0, uint32_t iv_word1, uint32_t iv_word2, uint32_t iv_word3,
    void* aad, uint64_t aad_bytes)
{
    using namespace sib;
    if (ciphertext == nullptr || key == nullptr || hash_subkey == nullptr || expected_tag == nullptr ||
        plaintext_output == nullptr || status_output == nullptr || bytes == 0 || (aad_bytes != 0 && aad == nullptr))
        return -1;
    if (bytes > kNoAllocMaxBytes || aad_bytes > kNoAllocMaxAad) {
        std::fprintf(stderr,
                     "secure_infer_aicpu_gcm_decrypt_verify_aad_noalloc_do: %llu payload / %llu AAD bytes exceed "
                     "the fixed scratch limit of %llu / %llu bytes\n",
                     static_cast<unsigned long long>(bytes), static_cast<unsigned long long>(aad_bytes),
                     static_cast<unsigned long long>(kNoAllocMaxBytes),
                     static_cast<unsigned long long>(kNoAllocMaxAad));
        return -2;
    }
    NoAllocScratch* scratch = noalloc_scratch();
    if (scratch == nullptr) return -1;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The arrival counter must start at zero; the kernel leaves it zero, but a
    // call that never completed would not, so clear it every time.
    if (cudaMemsetAsync(scratch->counters, 0, sizeof(scratch->counters), s) != cudaSuccess) return -1;
    if (launch_schedule(&scratch->sched, key, hash_subkey, true, s) != cudaSuccess) return -1;

    GcmRecord r{};
    r.op = kOpDecrypt;
    r.in = static_cast<const uint8_t*>(ciphertext);
    r.aad = static_cast<const uint8_t*>(aad_bytes ? aad : nullptr);
    r.aad_bytes = static_cast<uint32_t>(aad_bytes);
    r.tag_in = static_cast<const uint8_t*>(expected_tag);
    r.out = static_cast<uint8_t*>(plaintext_output);
    r.status = static_cast<uint32_t*>(status_output);
    r.count = bytes;
    r.iv[0] = iv_word0; r.iv[1] = iv_word1; r.iv[2] = iv_word2; r.iv[3] = iv_word3;
    const auto misaligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; };
    if (misaligned(ciphertext) || misaligned(plaintext_output)) r.flags |= kRecUnaligned;
    r.seg_first = 0;
    r.nseg = segments_for(bytes, r.aad_bytes);

    SegmentLaunch L{};
    L.sched = &scratch->sched;
    L.recs = nullptr;
    L.inl[0] = r;
    L.nrec = 1;
    L.total_segs = r.nseg;
    L.partials = scratch->partials;
    L.counters = scratch->counters;
    return launch_segments(L, true, s) == cudaSuccess ? 0 : -1;
}
