// Compile-only stand-in for the Metal framework header.  The reference's host
// files name Metal objects only as `id<Protocol>` return types of pipeline
// lookups; here `id<P>` is a plain pointer so that those declarations parse as
// C++ while every host generator body compiles unchanged.
#pragma once
struct MTLComputePipelineState;
template <class P>
using id = P*;
