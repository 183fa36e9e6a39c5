/*
 * fire_b200_alloc.h - device memory allocator of the fire_b200 library (B200, sm_100a).
 *
 * Replaces Fire's GPU DeviceAllocator (include/Fire/base/alloc.h:11-23 and :49-57,
 * src/base/alloc_cu.cpp:11-151, src/base/alloc.cpp:8-68): allocate / release a device
 * buffer, zero it, copy between host and device. Differences from the reference, all on
 * purpose: every call is thread-safe (the reference keeps unguarded std::maps), errors come
 * back as status codes (the reference CHECK-aborts or ignores CUDA errors), and blocks are
 * 256-byte aligned size-class blocks cached per device, so a released block is reused by
 * the next request of its class without a cudaMalloc. Status codes are those of fire_b200.h.
 */
#ifndef FIRE_B200_ALLOC_H
#define FIRE_B200_ALLOC_H

#include <stddef.h>

#include "fire_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* base::MemCpyKind (include/Fire/base/base.h:15-20), same values. */
enum {
    FIRE_B200_CPU2GPU = 0,
    FIRE_B200_CPU2CPU = 1,
    FIRE_B200_GPU2CPU = 2,
    FIRE_B200_GPU2GPU = 3
};

/* GPUAllocator::allocate (src/base/alloc_cu.cpp:11-79): a block of at least `bytes` on the
 * current device, 256-byte aligned, into *out. Requests are rounded up to a size class
 * (256 B granules up to 4 KiB, then four classes per power of two, 2 MiB granules above
 * 64 MiB); a cached free block of the class is reused, else the pool makes one with
 * cudaMalloc. FIRE_B200_ERR_NOMEM if the device has no room even after dropping the
 * device's cached free blocks. */
int fire_b200_device_alloc(size_t bytes, void** out);

/* GPUAllocator::release (src/base/alloc_cu.cpp:81-151): return a block to its device's
 * cache (NULL is a no-op). FIRE_B200_ERR_INVALID for a pointer this pool did not hand out
 * or one released twice (the reference CHECK-aborts). When the cached free bytes of a
 * device exceed 1 GiB, its free blocks are returned to CUDA. The caller must make sure no
 * queued GPU work still uses the block. */
int fire_b200_device_release(void* ptr);

/* DeviceAllocator::memset_zero (src/base/alloc.cpp:43-62) for device memory: asynchronous on
 * `stream` (NULL = legacy default stream); sync != 0 waits for the stream. */
int fire_b200_device_memset_zero(void* ptr, size_t bytes, void* stream, int sync);

/* DeviceAllocator::memcpy (src/base/alloc.cpp:8-41): kind is one of FIRE_B200_CPU2GPU ..
 * FIRE_B200_GPU2GPU; device copies are asynchronous on `stream`; sync != 0 waits for the
 * stream. CUDA errors are returned (the reference drops them). */
int fire_b200_device_memcpy(const void* src, void* dst, size_t bytes, int kind, void* stream, int sync);

/* Pool accounting of `device` (no reference counterpart): bytes held from CUDA, bytes in
 * blocks handed out, number of blocks handed out. */
int fire_b200_device_pool_stats(int device, size_t* reserved, size_t* in_use, size_t* live_blocks);

/* Return every cached free block of `device` to CUDA (no reference counterpart). */
int fire_b200_device_pool_trim(int device);

#ifdef __cplusplus
}
#endif
#endif /* FIRE_B200_ALLOC_H */
