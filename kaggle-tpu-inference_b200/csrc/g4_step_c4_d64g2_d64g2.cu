// Persistent decode-step kernel instantiation: rows up to 1024 elements
// (4 input chunks per lane), sliding layers head_dim 64 with 2 query heads per KV
// head, full layers head_dim 64 with 2 (per rank).
#include "g4_step.cuh"

G4_STEP_VARIANT(4, 64, 2, 64, 2)
