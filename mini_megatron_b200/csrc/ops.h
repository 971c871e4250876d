// Declarations of every kernel launcher exported by the extension.
#pragma once
#include "gemm_sm100.h"
