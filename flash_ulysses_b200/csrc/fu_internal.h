// Internal helpers shared by the C-ABI translation units.
#pragma once

namespace fu {
// Records a printf-style message for fu_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);
}  // namespace fu
