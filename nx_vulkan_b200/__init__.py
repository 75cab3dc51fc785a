"""nx_vulkan_b200 -- a B200 (sm_100a) implementation of nx_vulkan's hot path.

`vulkan` mirrors the reference's `Nx.Vulkan` API over the nxv_* C ABI that
libnxv_b200.so exports (include/nx_vulkan_shim.h); `compiler` lowers
elementwise chains to the fused op-tape kernel.  All tensor math runs on the
GPU; importing a submodule that needs the library fails loudly when it has
not been built.
"""
__all__ = ["vulkan", "compiler", "build"]
