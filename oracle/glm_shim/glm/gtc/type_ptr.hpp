// Empty stand-in: the reference includes this header but uses nothing from it.
#pragma once
#include "../glm.hpp"
