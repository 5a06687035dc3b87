#pragma once
#include "xrt_stub_types.h"
