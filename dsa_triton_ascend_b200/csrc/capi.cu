// Library-level entry points of libdsa_b200.so.
#include "dsa_b200.h"

extern "C" int dsa_version(void) { return (0 << 16) | 1; }
