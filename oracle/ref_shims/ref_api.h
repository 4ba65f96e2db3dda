/* Shared by the reference shims: every shim #includes one reference source
 * file where it lies and exports a few C entry points with default visibility
 * (everything else in the shim library is built hidden).  TEST INFRASTRUCTURE. */
#pragma once
#define REFAPI extern "C" __attribute__((visibility("default")))
