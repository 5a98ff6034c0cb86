// Instantiation shard 2 of the specialised (L, K) kernels (see pt_shapes.h).
#include "pt_registry.h"

PT_DEFINE_SHARD(2)
