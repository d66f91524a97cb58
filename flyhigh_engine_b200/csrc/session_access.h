// What the Stream layer (stream.cu) uses of a session beyond the C ABI: the same library, not exported.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

struct FhSession;
struct FhEngine;

namespace fhi {

// the message fh_last_error() returns on this thread
void set_error(const std::string& msg);
// the rgba8 frames of input slots a and b on the device, readable on stream `on` once this returns (it orders `on`
// after whatever wrote them); throws (an exception with the message) on a bad slot
void input_frames(FhSession* s, uint32_t a, uint32_t b, cudaStream_t on, const uint8_t** fa, const uint8_t** fb);
// frame width and height, network (internal) width and height, fine iterations and repair level of the session
void session_shape(const FhSession* s, int* w, int* h, int* iw, int* ih, int* k, int* repair);
// the stream the session's compute is ordered on (one-interval sessions: every pair and mid)
cudaStream_t compute_stream(FhSession* s);
// the rgba8 buffer of output slot `out`; output_written: the work issued on the compute stream so far is the last to
// write it (a read of the slot waits for that)
uint8_t* output_frame(FhSession* s, uint32_t out);
void output_written(FhSession* s, uint32_t out);
// the static age plane of the current pair (pitch in elements) and the protecting age; null / 0 without keep_static
void static_age(FhSession* s, const int16_t** age, int* pitch, float* min_age);
// whether the session was built with a protection mask (FhSessionOptions.protection_mask)
bool has_protection_mask(const FhSession* s);
// the work issued on the compute stream so far is the last to read input slots a and b (an upload into either waits
// for it): for readers on other streams that the compute stream has joined
void frames_read(FhSession* s, uint32_t a, uint32_t b);
// the CUDA device an engine runs on
int engine_device(const FhEngine* e);
// the network size a session of a w x h frame takes when the host gives none (options.rs:348-356)
void default_internal_size(int w, int h, int* iw, int* ih);

}  // namespace fhi
