// Stable LSD counting sort of (key, value) pairs, one digit of <= 8 bits per
// pass.  Each pass is a counting sort: per-segment shared-memory digit
// histograms (upsweep), a device scan of the digit-major histogram matrix, and
// a scatter whose in-segment ranks come from warp match-groups plus per-warp
// digit counters in shared memory (downsweep).  Ranks follow input order, so
// the sort is stable and its output is a pure function of its input.
#include "internal.h"
#include "oss_common.cuh"

namespace oss {
namespace {

constexpr int kRadixThreads = 256;
constexpr int kRadixWarps = kRadixThreads / 32;
constexpr int kRadixItems = 4;                                  // rounds of 32 per warp
constexpr int kWarpSpan = 32 * kRadixItems;                     // 128 items per warp
constexpr int kSegment = kRadixWarps * kWarpSpan;               // 1024 items per CTA
constexpr int kMaxDigits = 256;

__global__ void __launch_bounds__(kRadixThreads) k_radix_upsweep(const uint32_t* __restrict__ keys, int64_t n,
                                                                  int shift, uint32_t mask, int num_digits,
                                                                  int nseg, int32_t* __restrict__ counts) {
    __shared__ int32_t s_hist[kMaxDigits];
    for (int d = threadIdx.x; d < kMaxDigits; d += kRadixThreads) s_hist[d] = 0;
    __syncthreads();
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kSegment;
#pragma unroll
    for (int k = 0; k < kSegment / kRadixThreads; ++k) {
        const int64_t i = base + k * kRadixThreads + threadIdx.x;
        const bool valid = i < n;
        const uint32_t d = valid ? ((keys[i] >> shift) & mask) : 0xffffffffu;
        // warp-aggregated shared atomic: one add per distinct digit in the warp
        const unsigned peers = __match_any_sync(0xffffffffu, d);
        if (valid && (peers & lanemask_lt()) == 0) atomicAdd(&s_hist[d], __popc(peers));
    }
    __syncthreads();
    for (int d = threadIdx.x; d < num_digits; d += kRadixThreads) {
        counts[static_cast<int64_t>(d) * nseg + blockIdx.x] = s_hist[d];
    }
}

__global__ void __launch_bounds__(kRadixThreads) k_radix_downsweep(
    const uint32_t* __restrict__ keys_in, const int32_t* __restrict__ vals_in, int64_t n, int shift,
    uint32_t mask, int num_digits, int nseg, const int32_t* __restrict__ offsets,
    uint32_t* __restrict__ keys_out, int32_t* __restrict__ vals_out, int write_keys) {
    __shared__ int32_t s_cnt[kRadixWarps][kMaxDigits];
    for (int i = threadIdx.x; i < kRadixWarps * kMaxDigits; i += kRadixThreads) {
        (&s_cnt[0][0])[i] = 0;
    }
    __syncthreads();

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const unsigned lt = lanemask_lt();
    const int64_t wbase = static_cast<int64_t>(blockIdx.x) * kSegment + warp * kWarpSpan;

    uint32_t key[kRadixItems];
    int32_t val[kRadixItems];
    int32_t rank[kRadixItems];
    uint32_t dig[kRadixItems];
#pragma unroll
    for (int r = 0; r < kRadixItems; ++r) {
        const int64_t i = wbase + r * 32 + lane;
        const bool valid = i < n;
        key[r] = valid ? keys_in[i] : 0u;
        val[r] = valid ? vals_in[i] : 0;
        // invalid lanes carry digit kMaxDigits: they match only each other
        const uint32_t d = valid ? ((key[r] >> shift) & mask) : static_cast<uint32_t>(kMaxDigits);
        dig[r] = d;
        const unsigned peers = __match_any_sync(0xffffffffu, d);
        const int before = valid ? s_cnt[warp][d] : 0;
        __syncwarp();
        const unsigned lower = peers & lt;
        if (valid && lower == 0) s_cnt[warp][d] = before + __popc(peers);
        __syncwarp();
        rank[r] = before + __popc(lower);
    }
    __syncthreads();
    // digit-major prefix over warps, seeded with this segment's global digit offset
    for (int d = threadIdx.x; d < num_digits; d += kRadixThreads) {
        int32_t run = offsets[static_cast<int64_t>(d) * nseg + blockIdx.x];
#pragma unroll
        for (int wv = 0; wv < kRadixWarps; ++wv) {
            const int32_t c = s_cnt[wv][d];
            s_cnt[wv][d] = run;
            run += c;
        }
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kRadixItems; ++r) {
        const int64_t i = wbase + r * 32 + lane;
        if (i < n) {
            const int32_t pos = s_cnt[warp][dig[r]] + rank[r];
            vals_out[pos] = val[r];
            if (write_keys) keys_out[pos] = key[r];
        }
    }
}

struct RadixPlan {
    int passes;
    int bits[4];
    int shift[4];
};

RadixPlan make_plan(uint32_t key_limit) {
    RadixPlan p{};
    int total_bits = 0;
    while (total_bits < 32 && (key_limit >> total_bits) != 0u) ++total_bits;
    p.passes = (total_bits + 7) / 8;
    int shift = 0;
    for (int i = 0; i < p.passes; ++i) {
        const int remaining = total_bits - shift;
        const int b = (remaining + (p.passes - i) - 1) / (p.passes - i);
        p.bits[i] = b;
        p.shift[i] = shift;
        shift += b;
    }
    return p;
}

}  // namespace

int64_t radix_scratch_bytes(int64_t n, uint32_t key_limit) {
    const RadixPlan p = make_plan(key_limit);
    const int64_t nseg = div_up(n, kSegment);
    int64_t bytes = 0;
    bytes += arena_bytes(n, sizeof(uint32_t));  // ping-pong keys
    bytes += arena_bytes(n, sizeof(int32_t));   // ping-pong vals
    bytes += arena_bytes(static_cast<int64_t>(kMaxDigits) * nseg, sizeof(int32_t));
    bytes += scan_scratch_bytes(static_cast<int64_t>(kMaxDigits) * nseg);
    (void)p;
    return bytes;
}

cudaError_t radix_sort_pairs(uint32_t* keys, int32_t* vals, int64_t n, uint32_t key_limit,
                             int32_t* vals_out, void* scratch, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    const RadixPlan plan = make_plan(key_limit);
    if (plan.passes == 0) {  // all keys are 0: input order is the sorted order
        return cudaMemcpyAsync(vals_out, vals, n * sizeof(int32_t), cudaMemcpyDeviceToDevice, stream);
    }
    const int64_t nseg = div_up(n, kSegment);
    Arena arena{static_cast<char*>(scratch), radix_scratch_bytes(n, key_limit), 0};
    uint32_t* keys_alt = arena.take<uint32_t>(n);
    int32_t* vals_alt = arena.take<int32_t>(n);
    int32_t* counts = arena.take<int32_t>(static_cast<int64_t>(kMaxDigits) * nseg);
    void* scan_scratch = arena.base + arena.used;

    uint32_t* kin = keys;
    int32_t* vin = vals;
    uint32_t* kout = keys_alt;
    int32_t* vout = vals_alt;
    for (int pass = 0; pass < plan.passes; ++pass) {
        const int num_digits = 1 << plan.bits[pass];
        const uint32_t mask = static_cast<uint32_t>(num_digits - 1);
        const bool last = pass == plan.passes - 1;
        k_radix_upsweep<<<static_cast<unsigned>(nseg), kRadixThreads, 0, stream>>>(
            kin, n, plan.shift[pass], mask, num_digits, static_cast<int>(nseg), counts);
        cudaError_t err = scan_exclusive_i32(counts, counts, static_cast<int64_t>(num_digits) * nseg, false,
                                             nullptr, scan_scratch, stream);
        if (err != cudaSuccess) return err;
        int32_t* dst_vals = last ? vals_out : vout;
        k_radix_downsweep<<<static_cast<unsigned>(nseg), kRadixThreads, 0, stream>>>(
            kin, vin, n, plan.shift[pass], mask, num_digits, static_cast<int>(nseg), counts, kout, dst_vals,
            last ? 0 : 1);
        err = cudaGetLastError();
        if (err != cudaSuccess) return err;
        // next pass reads what this one wrote
        uint32_t* kt = kin;
        kin = kout;
        kout = kt;
        int32_t* vt = vin;
        vin = dst_vals;
        vout = vt;
    }
    return cudaGetLastError();
}

}  // namespace oss
