// ABI-wide entry points: version and the per-thread last-error message.
#include "capi_common.cuh"

extern "C" int ttt_abi_version(void) { return 10000; }

extern "C" const char* ttt_last_error(void) { return ttt::last_error_buffer(); }
