// bootstrap/bootstrap.hpp -- the include path the reference's programs use for the process
// bootstrap; the class itself is gicc::Bootstrap in gicc/bootstrap.hpp.
#pragma once

#include "gicc/bootstrap.hpp"
