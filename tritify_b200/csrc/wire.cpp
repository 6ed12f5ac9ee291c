// The activation interchange format: IntTensor::to_bytes / IntTensor::from_bytes (kt-core/src/tensor.rs:51-100).
//
// Little-endian, fixed widths, no padding:
//   u32 ndim | ndim x u64 shape | i64 scale.mant | i32 scale.shift | u64 ndata | ndata x i32 codes
// The reference passes an activation between workers in this form so that the receiver continues the same exact
// computation; this library reads and writes it byte for byte, so its expert outputs (and layer inputs and outputs)
// can cross a host boundary to or from the reference's workers. Bytes are assembled one at a time, so the result
// does not depend on the host's byte order.

#include <stddef.h>
#include <stdint.h>

#include "ktmoe.h"

namespace {

void put_u32(uint8_t* p, uint32_t v) {
    for (int i = 0; i < 4; ++i) p[i] = (uint8_t)(v >> (8 * i));
}
void put_u64(uint8_t* p, uint64_t v) {
    for (int i = 0; i < 8; ++i) p[i] = (uint8_t)(v >> (8 * i));
}
uint32_t get_u32(const uint8_t* p) {
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) v |= (uint32_t)p[i] << (8 * i);
    return v;
}
uint64_t get_u64(const uint8_t* p) {
    uint64_t v = 0;
    for (int i = 0; i < 8; ++i) v |= (uint64_t)p[i] << (8 * i);
    return v;
}

// 4 + 8·ndim + 8 + 4 + 8 + 4·ndata, or 0 when it does not fit in 64 bits.
uint64_t frame_bytes(uint64_t ndim, uint64_t ndata) {
    if (ndim > (UINT64_MAX - 24) / 8) return 0;
    const uint64_t head = 24 + 8 * ndim;
    if (ndata > (UINT64_MAX - head) / 4) return 0;
    return head + 4 * ndata;
}

}  // namespace

extern "C" {

int ktmoe_wire_size(int32_t ndim, int64_t ndata, uint64_t* bytes) {
    if (ndim < 0 || ndata < 0 || !bytes) return KTMOE_ERR_ARG;
    const uint64_t n = frame_bytes((uint64_t)ndim, (uint64_t)ndata);
    if (n == 0) return KTMOE_ERR_ARG;
    *bytes = n;
    return KTMOE_OK;
}

int ktmoe_wire_encode(const int32_t* data, int64_t ndata, const int64_t* shape, int32_t ndim, ktmoe_scale scale,
                      uint8_t* out, uint64_t cap, uint64_t* written) {
    if (ndim < 0 || ndata < 0 || (ndim > 0 && !shape) || (ndata > 0 && !data) || !out || !written) return KTMOE_ERR_ARG;
    for (int32_t i = 0; i < ndim; ++i)
        if (shape[i] < 0) return KTMOE_ERR_ARG;
    const uint64_t n = frame_bytes((uint64_t)ndim, (uint64_t)ndata);
    if (n == 0 || n > cap) return KTMOE_ERR_ARG;
    uint8_t* p = out;
    put_u32(p, (uint32_t)ndim);
    p += 4;
    for (int32_t i = 0; i < ndim; ++i, p += 8) put_u64(p, (uint64_t)shape[i]);
    put_u64(p, (uint64_t)scale.mant);
    p += 8;
    put_u32(p, (uint32_t)scale.shift);
    p += 4;
    put_u64(p, (uint64_t)ndata);
    p += 8;
    for (int64_t i = 0; i < ndata; ++i, p += 4) put_u32(p, (uint32_t)data[i]);
    *written = n;
    return KTMOE_OK;
}

int ktmoe_wire_decode(const uint8_t* b, uint64_t len, int32_t* ndim, int64_t* shape, int32_t shape_cap,
                      ktmoe_scale* scale, int64_t* ndata, int32_t* data, int64_t data_cap, uint64_t* consumed) {
    if (!b || !ndim || !scale || !ndata || !consumed || shape_cap < 0 || data_cap < 0) return KTMOE_ERR_ARG;
    if (len < 4) return KTMOE_ERR_ARG;
    const uint64_t nd = get_u32(b);
    if (nd > (uint64_t)INT32_MAX || len < 24 + 8 * nd) return KTMOE_ERR_ARG;
    const uint8_t* p = b + 4;
    if ((uint64_t)shape_cap < nd && shape) return KTMOE_ERR_ARG;
    for (uint64_t i = 0; i < nd; ++i, p += 8) {
        const uint64_t s = get_u64(p);
        if (s > (uint64_t)INT64_MAX) return KTMOE_ERR_ARG;
        if (shape) shape[i] = (int64_t)s;
    }
    scale->mant = (int64_t)get_u64(p);
    p += 8;
    scale->shift = (int32_t)get_u32(p);
    p += 4;
    const uint64_t n = get_u64(p);
    p += 8;
    const uint64_t total = frame_bytes(nd, n);
    if (total == 0 || len < total || n > (uint64_t)INT64_MAX) return KTMOE_ERR_ARG;
    *ndim = (int32_t)nd;
    *ndata = (int64_t)n;
    *consumed = total;
    if (data) {
        if ((uint64_t)data_cap < n) return KTMOE_ERR_ARG;
        for (uint64_t i = 0; i < n; ++i, p += 4) data[i] = (int32_t)get_u32(p);
    }
    return KTMOE_OK;
}

}  // extern "C"
