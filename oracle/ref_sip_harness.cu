// Test-only harness around the reference SIP kernel (AB-Attention csrc/sip.cu).
//
// ORACLE INFRASTRUCTURE: compiled by oracle/build_ref.py into oracle/_ref/ and
// used only by tests, smoke() and bench.py's CPU-baseline leg as a checker.
// The reference source is included where it lies; `sip_cuda`
// (csrc/sip.cu:170-199) is exported through ref_bindings.cpp unchanged.
#include "sip.cu"
