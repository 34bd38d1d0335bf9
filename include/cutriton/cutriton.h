#pragma once

// Aggregate header of the public C++17 API (same include set as the
// reference's include/cutriton/cutriton.h:5-20).
#include "cutriton/core/buffer.h"
#include "cutriton/core/device.h"
#include "cutriton/core/status.h"
#include "cutriton/core/tensor.h"
#include "cutriton/backend/backend.h"
#include "cutriton/compiler/compiler.h"
#include "cutriton/ir/graph.h"
#include "cutriton/ir/fusion.h"
#include "cutriton/ir/op_schema.h"
#include "cutriton/ir/pass.h"
#include "cutriton/runtime/engine.h"
#include "cutriton/runtime/executable_plan.h"
#include "cutriton/runtime/memory_planner.h"
#include "cutriton/runtime/profiler.h"
#include "cutriton/runtime/shape_profile.h"
#include "cutriton/runtime/tuning.h"
