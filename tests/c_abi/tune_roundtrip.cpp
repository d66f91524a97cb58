// The conv autotune table's text format (flyhigh_engine_b200/csrc/tune.hpp), checked on the host: prints one line per
// check, "ok <name>" or "FAIL <name>", and exits non-zero on a failure. Built and run by tests/test_c_abi.py.
#include <cstdio>

#include "tune.hpp"

static int failures = 0;
static void check(bool ok, const char* name) {
    printf("%s %s\n", ok ? "ok" : "FAIL", name);
    if (!ok) failures++;
}

int main() {
    // the reference's own case (crates/flyhigh-engine/tests/defaults.rs:55-63): two good lines among malformed ones
    const char* text = "96,96,60,108,1=18\nnot a line\n36,36,180,320,1=2\n1,2,3=4\n48,48,60,108,1=x\n";
    fhtune::Table t = fhtune::parse(text);
    check(t.size() == 2, "two entries");
    check(t.count(fhtune::Key{96, 96, 60, 108, 1}) && t[fhtune::Key{96, 96, 60, 108, 1}] == 18, "value 18");
    check(fhtune::parse(fhtune::format(t)) == t, "round trip");
    check(fhtune::format(t) == "36,36,180,320,1=2\n96,96,60,108,1=18", "sorted lines");
    check(fhtune::parse("").empty() && fhtune::parse("garbage").empty(), "empty and garbage");
    check(fhtune::parse("1,2,3,4,5=256\n1,2,3,4,5=-1\n1,2,3,4,5,6=1\n").empty(), "out of range and extra fields");
    check(fhtune::parse(" 48 , 48 , 60 , 108 , 1 = 33 \r\n").at(fhtune::Key{48, 48, 60, 108, 1}) == 33, "spaces");
    // this library's candidate bytes
    check(fhtune::valid(fhtune::mma(1)) && fhtune::valid(fhtune::mma(2)) && fhtune::valid(fhtune::mma(4)) &&
              fhtune::valid(fhtune::mma(0)) && fhtune::valid(fhtune::KERNEL_UMMA) &&
              fhtune::valid(fhtune::UMMA_PERSISTENT) && fhtune::UMMA_PERSISTENT == 18,
          "candidates valid");
    check(!fhtune::valid(0x22) && !fhtune::valid(0) && !fhtune::valid(0x31) && !fhtune::valid(3), "others refused");
    check(fhtune::name(fhtune::mma(2)) == "mma.sync/wm2" && fhtune::name(fhtune::KERNEL_UMMA) == "tcgen05" &&
              fhtune::name(fhtune::UMMA_PERSISTENT) == "tcgen05/persistent",
          "names");
    const std::string f = fhtune::file_name("/tmp/x", "NVIDIA B200", 12090);
    check(f.rfind("/tmp/x/tune-10de-", 0) == 0 && f.size() > 30 && f.substr(f.size() - 16) == "-f16-tc-b200.txt",
          "file name");
    return failures ? 1 : 0;
}
