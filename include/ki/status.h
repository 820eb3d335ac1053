/*
 * ki/status.h -- bits that device-side code latches into a 32-bit status word with atomicOr when a
 * bounded wait runs out or a value is inconsistent.  libki_b200 reads its contexts' status words in
 * ki_ctx_check and reports KI_ERR_TIMEOUT / KI_ERR_CUDA; kernels written against the device headers
 * in this directory can use their own word.
 */
#ifndef KI_STATUS_H
#define KI_STATUS_H

#include <stdint.h>

enum : uint32_t {
    KI_DEV_TIMEOUT = 1u,   /* a bounded wait ran out */
    KI_DEV_BAD_STATE = 2u  /* a kernel saw an impossible value (e.g. a corrupt tile flag) */
};

#endif /* KI_STATUS_H */
