/* The library's public header, one directory up from the Swift package (the repository root). */
#include "../../../../include/va_cuda.h"
