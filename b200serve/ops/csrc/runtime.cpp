// Process-wide switches of the extension.
#include <cstdlib>
#include <cstring>

namespace b200 {

static int g_pdl = -1;

bool pdl_enabled() {
  if (g_pdl < 0) {
    const char* v = std::getenv("B200_PDL");
    g_pdl = (v && (std::strcmp(v, "0") == 0)) ? 0 : 1;   // on unless B200_PDL=0
  }
  return g_pdl != 0;
}

void set_pdl(bool on) { g_pdl = on ? 1 : 0; }

}  // namespace b200
