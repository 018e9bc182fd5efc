// Drives kestrel_b200/csrc/expert_cache.h from a text script on stdin (used
// by tests/test_expert_cache.py, on the CPU). One command per line:
//   config <capacity> <scratch> <policy 0=LFRU 1=LRU> [<spec slots>]
//   demand <layer> <n> <e1> ... <en>   -> "D <slots...> | <expert:slot loads...> | <wait slots...>" or "D fail"
//   prefetch <layer> <n> <e1> ... <en> -> "P <expert:slot loads...>"
//   done <slot>                        (a prefetch copy landed)
//   decay
//   slot <layer> <e>                   -> "S <slot or -1>"
//   heat <layer> <e>                   -> "H <heat> <last>"
//   stats                              -> "T <requests hits late misses scratch_loads prefetch_issued
//                                          prefetch_used prefetch_wasted evictions forced cached spec_pauses>"
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

#include "expert_cache.h"

int main() {
  kc::ExpertCache c;
  std::string line;
  std::vector<kc::ExpertCache::Load> loads;
  std::vector<int> waits;
  while (std::getline(std::cin, line)) {
    std::istringstream in(line);
    std::string cmd;
    if (!(in >> cmd)) continue;
    if (cmd == "config") {
      int cap, scr, pol, spec = 0;
      in >> cap >> scr >> pol >> spec;
      c.configure(cap, scr, spec, pol ? kc::ExpertPolicy::Lru : kc::ExpertPolicy::Lfru);
    } else if (cmd == "demand" || cmd == "prefetch") {
      int layer, n;
      in >> layer >> n;
      std::vector<int> e(n), slot(n, -1);
      for (int& x : e) in >> x;
      if (cmd == "prefetch") {
        c.prefetch(layer, e.data(), n, loads);
        std::cout << "P";
        for (auto& ld : loads) std::cout << ' ' << ld.expert << ':' << ld.slot;
        std::cout << '\n';
        continue;
      }
      if (!c.demand(layer, e.data(), n, slot.data(), loads, waits)) {
        std::cout << "D fail\n";
        continue;
      }
      std::cout << "D";
      for (int s : slot) std::cout << ' ' << s;
      std::cout << " |";
      for (auto& ld : loads) std::cout << ' ' << ld.expert << ':' << ld.slot;
      std::cout << " |";
      for (int s : waits) std::cout << ' ' << s;
      std::cout << '\n';
    } else if (cmd == "done") {
      int s;
      in >> s;
      c.mark_done(s);
    } else if (cmd == "decay") {
      c.decay();
    } else if (cmd == "slot") {
      int layer, e;
      in >> layer >> e;
      std::cout << "S " << c.slot_of(layer, e) << '\n';
    } else if (cmd == "heat") {
      int layer, e;
      in >> layer >> e;
      std::cout << "H " << c.heat(layer, e) << ' ' << c.last(layer, e) << '\n';
    } else if (cmd == "stats") {
      const kc::ExpertCacheStats& s = c.stats();
      std::cout << "T " << s.requests << ' ' << s.hits << ' ' << s.late << ' ' << s.misses << ' ' << s.scratch_loads
                << ' ' << s.prefetch_issued << ' ' << s.prefetch_used << ' ' << s.prefetch_wasted << ' '
                << s.evictions << ' ' << s.forced << ' ' << c.cached() << ' ' << s.spec_pauses << '\n';
    } else {
      std::cerr << "unknown command " << cmd << '\n';
      return 2;
    }
  }
  return 0;
}
