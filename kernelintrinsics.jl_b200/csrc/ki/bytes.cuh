// ki/bytes.cuh -- 16-byte word helpers shared by the byte copies (copy.cu, copy2d.cu).
#pragma once

#include <cstdint>

namespace ki {

// The 16 bytes that start 4*WS + sh/8 bytes into the 32-byte pair (lo, hi): a source that is
// misaligned against its destination still moves as aligned 16-byte loads.
template <int WS>
__device__ __forceinline__ uint4 realign(const uint4& lo, const uint4& hi, unsigned sh) {
    const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
    uint4 r;
    r.x = __funnelshift_r(w[WS + 0], w[WS + 1], sh);
    r.y = __funnelshift_r(w[WS + 1], w[WS + 2], sh);
    r.z = __funnelshift_r(w[WS + 2], w[WS + 3], sh);
    r.w = __funnelshift_r(w[WS + 3], w[WS + 4], sh);
    return r;
}

// The next lane's 16-byte word (lane 31 gets its own back).
__device__ __forceinline__ uint4 shfl_down_u4(const uint4& v) {
    uint4 r;
    r.x = __shfl_down_sync(0xffffffffu, v.x, 1);
    r.y = __shfl_down_sync(0xffffffffu, v.y, 1);
    r.z = __shfl_down_sync(0xffffffffu, v.z, 1);
    r.w = __shfl_down_sync(0xffffffffu, v.w, 1);
    return r;
}

}  // namespace ki
