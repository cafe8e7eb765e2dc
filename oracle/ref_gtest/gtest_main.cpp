// main() of the runnable GoogleTest stand-in (ref_gtest/gtest/gtest.h): runs
// every registered TEST in registration order, or those whose "Suite.Name"
// contains the first argument, printing GoogleTest-style lines. Exit status 0
// when every test that ran passed, 1 otherwise. Test infrastructure only.
#include <gtest/gtest.h>

#include <cstring>
#include <exception>

int main(int argc, char **argv)
{
    const char *filter = argc > 1 ? argv[1] : nullptr;
    int ran = 0, failed = 0;
    std::vector<std::string> failed_names;
    for (const auto &t : ref_gtest::registry())
    {
        std::string full = std::string(t.suite) + "." + t.name;
        if (filter && !std::strstr(full.c_str(), filter))
            continue;
        std::printf("[ RUN      ] %s\n", full.c_str());
        std::fflush(stdout);
        ref_gtest::failures_in_current_test() = 0;
        try
        {
            t.fn();
        }
        catch (const std::exception &e)
        {
            ++ref_gtest::failures_in_current_test();
            std::printf("unexpected exception: %s\n", e.what());
        }
        ++ran;
        if (ref_gtest::failures_in_current_test())
        {
            ++failed;
            failed_names.push_back(full);
            std::printf("[  FAILED  ] %s\n", full.c_str());
        }
        else
            std::printf("[       OK ] %s\n", full.c_str());
        std::fflush(stdout);
    }
    std::printf("[==========] %d tests ran.\n[  PASSED  ] %d tests.\n", ran, ran - failed);
    for (const auto &n : failed_names)
        std::printf("[  FAILED  ] %s\n", n.c_str());
    return failed ? 1 : 0;
}
