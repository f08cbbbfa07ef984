// megakernel.cuh — persistent batch-1 decode step (filled in below).
#pragma once
struct MegaState { int ready = 0; };
inline void mega_free(MegaState & m) { m.ready = 0; }
