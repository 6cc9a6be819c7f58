#pragma once
// Bounded spin-waits for device code.
//
// The reference's device waits spin forever (device.cuh:110-118,
// device_primitives.cuh:117-150, sg_device_primitives.cuh:28-243).  Every wait in
// this library gives up after a time limit measured on %globaltimer, counts the
// give-up in a host-visible word, and returns false, so a missing producer or
// consumer turns into an error the host can read instead of a hung GPU.

#include <cstdint>

#include "gfd/pull.cuh"

#ifndef GFD_DEVICE_WAIT_LIMIT_NS
#define GFD_DEVICE_WAIT_LIMIT_NS 10000000000ull  // 10 s
#endif

namespace gfd {
namespace wait {

__device__ __forceinline__ uint64_t now() { return gfd::pull::globaltimer_ns(); }

// Spin/backoff step: tight for the first 64 polls, then __nanosleep 100 ns, then 1 us.
__device__ __forceinline__ void backoff(uint32_t& polls) {
    ++polls;
    if (polls > 64) __nanosleep(polls < 256 ? 100 : 1000);
}

__device__ __forceinline__ bool expired(uint64_t t0, uint64_t limit_ns) {
    return now() - t0 > (limit_ns ? limit_ns : GFD_DEVICE_WAIT_LIMIT_NS);
}

__device__ __forceinline__ uint64_t load_acquire_sys(const volatile uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t load_acquire_sys(const volatile uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Relaxed system-scope loads: several may be in flight at once (acquire loads wait for
// one another); pair them with a fence to acquire.
__device__ __forceinline__ uint64_t load_relaxed_sys(const volatile uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t load_relaxed_sys(const volatile uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Monotonic publication of a counter to a host-visible word: one atomic max whose
// result is not used, so the issuing thread does not wait for the round trip.
__device__ __forceinline__ void publish_max(volatile uint64_t* host_word, unsigned long long v) {
    atomicMax(reinterpret_cast<unsigned long long*>(const_cast<uint64_t*>(host_word)), v);
}

// Records a give-up in a host-visible 32-bit counter (may be null).
__device__ __forceinline__ void note_timeout(volatile uint32_t* counter) {
    if (counter != nullptr) atomicAdd(const_cast<uint32_t*>(counter), 1u);
    __threadfence_system();
}

}  // namespace wait
}  // namespace gfd
