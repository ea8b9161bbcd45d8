// Umbrella header: host entry points of every mdl_b200 kernel family.
#pragma once

#include "gemm.h"
