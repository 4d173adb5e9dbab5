// Parity oracle (test infrastructure, see oracle.h): b2World::SolveTOI (toi.py).
#include "oracle.h"

namespace orc {
void solve_toi(const Model &m, World &w, const goib2d_settings &s, float dt) {
    (void)dt;
    if (w.C == 0 || m.P == 0) return;
    if (s.unity_toi && m.d->toi_bodies) {
        bool any = false;
        for (int b = 0; b < m.B; ++b) any = any || m.d->toi_bodies[b];
        if (!any) return;
    }
    // TODO: full SolveTOI
}
}  // namespace orc
