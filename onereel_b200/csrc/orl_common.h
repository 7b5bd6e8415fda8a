// Internal header: the public C ABI plus C++ aliases shared by the .cu files.
#pragma once

#include "../../include/onereel_b200.h"

namespace orl {
using AttnWork = orl_attn_work;
using CopyRun = orl_copy_run;
static_assert(sizeof(AttnWork) == 32, "work item layout");
static_assert(sizeof(CopyRun) == 32, "copy run layout");
}  // namespace orl
