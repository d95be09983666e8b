// Stand-in (test infrastructure; see ggml.h): the graph allocator type of
// the reference's plan_t.
#pragma once
#include "ggml.h"

typedef struct ggml_gallocr *ggml_gallocr_t;
