#pragma once
// Stand-in: see NvInferRuntime.h in this folder.
#include "NvInferRuntime.h"
