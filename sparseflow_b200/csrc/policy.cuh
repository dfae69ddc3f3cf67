// Host-side access to the path policy set through sf_set_path_policy.
#pragma once
#include "../../include/sparseflow_b200.h"

namespace sf {
long long policy(int key);
}  // namespace sf
