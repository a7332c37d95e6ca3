// Device-side decode state shared by the engine kernels (one per engine, in HBM).
#pragma once

namespace jinf {

// Device error codes written to DeviceState::error (first error wins).
enum DeviceError { DEV_OK = 0, DEV_ERR_TIMEOUT = 1 };

struct DeviceState {
    int pos;                  // position of the token being decoded (= n_past before the step)
    int token;                // input token id of the current step
    unsigned long long best;  // packed (ordered logit << 32 | ~index) argmax of the last LM head
    int argmax_token;         // decoded argmax of the last step
    int error;                // first device-side error code (DEV_OK = none)
    unsigned int attn_count[64];  // split-K arrival counters of the attention kernel (self-resetting)
};

}  // namespace jinf
