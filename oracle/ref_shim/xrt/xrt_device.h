// Empty stand-ins so include/xdna/dma_streamer.h (which includes the XRT
// headers unconditionally) compiles in a build without XRT.  Nothing from XRT
// is used unless XDNA_WITH_XRT is defined, which this recipe never does.
#pragma once
namespace xrt {
class device {};
class bo {};
}  // namespace xrt
