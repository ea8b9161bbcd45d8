// Umbrella header: host entry points of every mdl_b200 kernel family.
#pragma once

#include "attention.h"
#include "attn_simt.h"
#include "comm.h"
#include "embedding.h"
#include "fmha.h"
#include "gemm.h"
#include "misc.h"
#include "norm.h"
#include "sqa.h"
