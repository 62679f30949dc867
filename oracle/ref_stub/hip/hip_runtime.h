// Test-infrastructure stub (oracle only). The reference's host headers include
// <hip/hip_runtime.h> and name hipStream_t in one declaration; this is the whole of
// what the host-side code that the oracle compiles needs from HIP.
#pragma once
typedef struct ihipStream_t* hipStream_t;
