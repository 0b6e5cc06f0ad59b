// See xrt_device.h in this directory.
#pragma once
#include "xrt_device.h"
