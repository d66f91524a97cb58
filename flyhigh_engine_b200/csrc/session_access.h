// What the Stream layer (stream.cu) uses of a session beyond the C ABI: the same library, not exported.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

struct FhSession;

namespace fhi {

// the message fh_last_error() returns on this thread
void set_error(const std::string& msg);
// the rgba8 frames of input slots a and b on the device, readable on stream `on` once this returns (it orders `on`
// after whatever wrote them); throws (an exception with the message) on a bad slot
void input_frames(FhSession* s, uint32_t a, uint32_t b, cudaStream_t on, const uint8_t** fa, const uint8_t** fb);
// frame width and height, network (internal) width and height, fine iterations and repair level of the session
void session_shape(const FhSession* s, int* w, int* h, int* iw, int* ih, int* k, int* repair);

}  // namespace fhi
