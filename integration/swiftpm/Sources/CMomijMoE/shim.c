/* SwiftPM needs one source file in a C target; the code lives in
 * libmomij_moe.so, declared by include/momij_moe.h. */
#include "momij_moe.h"
