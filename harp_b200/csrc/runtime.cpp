// placeholder, replaced by the host runtime
#include <ATen/ATen.h>
