// Command capture and CUDA-graph replay for backend-cuda (see slc_set_capture
// in include/starlight_cuda.h).
#include "device_internal.h"

struct CaptureState {
    bool enabled = false;
};

extern "C" int slc_set_capture(slc_device *d, int enabled) {
    if (!d) return SLC_ERR_EXECUTION;
    (void)enabled;
    return slc_fail(d, SLC_ERR_UNIMPLEMENTED, "command capture is not available in this build");
}

int flush_capture(slc_device *) { return SLC_OK; }
void release_capture(slc_device *d) {
    delete d->capture;
    d->capture = nullptr;
}
int capture_record(slc_device *, const slc_op *, const slc_buffer_ref *, const slc_value *,
                   uint64_t, const slc_buffer_ref *, const slc_value *, uint64_t,
                   const uint32_t *, uint64_t) {
    return 0;
}
