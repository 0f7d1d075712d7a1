// Allocation-free forward trace: sdfoam_trace_forward_noalloc.
//
// The regular entry points take their scratch (the cell records) from the
// caller.  Some callers cannot provide it: code that reaches this library
// through the C ABI from a runtime with no device allocator of its own (a
// Go / Java / Rust host, a plugin inside another renderer), and frame loops
// such as an interactive viewer that must not call cudaMalloc / cudaFree per
// frame because those calls can synchronise the whole device and stall the
// frame.  For them this entry point keeps the cell records in one file-scope
// device array of fixed size and allocates nothing.
//
// Limits and rules:
//   * the array holds kNoallocCellsBytes = 64 MiB on every GPU that loads the
//     library, until the process exits;
//   * foams whose cell records need more (sdfoam_cells_bytes) are rejected
//     with SDFOAM_ERR_INVALID; at SH degree 3 and the usual Delaunay mean
//     degree of ~15 (256-byte site record + 15 x 16-byte face records +
//     18 x 8-byte plane slots) that is about 100k sites;
//   * every call shares the array and leaves the last call's records in it;
//     calls whose GPU work overlaps (different streams, or different host
//     threads on one device) race on it and must be serialised by the caller;
//   * nothing in the array has to start at zero: the build writes every
//     record the walk reads;
//   * every call resolves the array's device address with
//     cudaGetSymbolAddress for the current device (no allocation, a few
//     microseconds), so the address stays right after cudaDeviceReset or a
//     new primary context; the first call on a device also loads the
//     library's module there, so make it before any stream capture.
#include <string>

#include "foam_internal.h"

namespace {

constexpr size_t kNoallocCellsBytes = size_t(64) << 20;

// Device storage for the cell records.  In host code this name is only a
// host-side stand-in for the symbol, not a device address: the kernels get
// the address resolved by cudaGetSymbolAddress below.
__device__ __align__(256) unsigned char g_noalloc_cells[kNoallocCellsBytes];

// The device address of g_noalloc_cells on the current device, resolved
// with that device current.
int noalloc_scratch(void **out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        sdfoam_b200::set_last_error(std::string("sdfoam_trace_forward_noalloc: cudaGetDevice: ") +
                                    cudaGetErrorString(e));
        return SDFOAM_ERR_CUDA;
    }
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_cells);
    if (e != cudaSuccess || p == nullptr) {
        sdfoam_b200::set_last_error(std::string("sdfoam_trace_forward_noalloc: cudaGetSymbolAddress: ") +
                                    cudaGetErrorString(e));
        return SDFOAM_ERR_CUDA;
    }
    *out = p;
    return SDFOAM_OK;
}

}  // namespace

extern "C" int sdfoam_trace_forward_noalloc(const sdfoam_foam *foam, const sdfoam_trace_settings *settings,
                                            const sdfoam_forward_io *io, sdfoam_stream_t stream) {
    if (!foam) {
        sdfoam_b200::set_last_error("foam is NULL");
        return SDFOAM_ERR_INVALID;
    }
    const size_t need = sdfoam_cells_bytes(foam->num_points, foam->adjacency_size, foam->sh_degree);
    if (need == 0) {
        // an SH degree or foam size that no entry point takes: the same
        // code and message as sdfoam_build_cells
        return sdfoam_build_cells(foam, nullptr, 0, stream);
    }
    if (need > kNoallocCellsBytes) {
        sdfoam_b200::set_last_error(
            "sdfoam_trace_forward_noalloc: the foam needs " + std::to_string(need) +
            " bytes of cell records but the static scratch holds " + std::to_string(kNoallocCellsBytes) +
            " bytes; use sdfoam_build_cells + sdfoam_trace_forward with a caller-owned workspace");
        return SDFOAM_ERR_INVALID;
    }
    void *cells = nullptr;
    if (int rc = noalloc_scratch(&cells)) return rc;
    if (int rc = sdfoam_build_cells(foam, cells, kNoallocCellsBytes, stream)) return rc;
    return sdfoam_trace_forward(foam, cells, settings, io, stream);
}
