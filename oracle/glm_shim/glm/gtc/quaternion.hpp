// Part of the GLM API stand-in (TEST INFRASTRUCTURE ONLY); everything lives in glm.hpp.
#pragma once
#include "../glm.hpp"
