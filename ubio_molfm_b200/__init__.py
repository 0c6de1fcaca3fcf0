"""B200-native E2Former-V2 sparse equivariant attention, its graph builder and the model around it."""
import os

# An MD run rebuilds its neighbour graph every step, so the edge tensors change size from step to step;
# near the device's capacity the caching allocator's fixed-size segments then fragment, and it frees
# and re-maps memory (a device-wide synchronisation, measured at up to 1.4 s on a 0.4 s step).  Growable
# segments avoid that.  This takes effect only if set before the process first allocates device memory
# (import this package first, or set PYTORCH_CUDA_ALLOC_CONF yourself).
os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
