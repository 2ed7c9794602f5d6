// main() for the gtest-compatible harness in gtest/gtest.h: runs every
// registered TEST in registration order (optionally those whose
// "Suite.Name" contains the --gtest_filter= text), prints gtest-style
// progress lines, and exits 1 if any test failed.
#include <exception>
#include <iostream>
#include <string>

#include "gtest/gtest.h"

int main(int argc, char** argv) {
    std::string filter;
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        if (a.rfind("--gtest_filter=", 0) == 0)
            filter = a.substr(15);
    }
    int run = 0, failed = 0;
    for (const auto& c : ttgt::registry()) {
        const std::string full = std::string(c.suite) + "." + c.name;
        if (!filter.empty() && full.find(filter) == std::string::npos)
            continue;
        ++run;
        std::cout << "[ RUN      ] " << full << std::endl;
        ttgt::current_failures() = 0;
        try {
            c.fn();
        } catch (const std::exception& e) {
            std::cout << "uncaught exception: " << e.what() << std::endl;
            ++ttgt::current_failures();
        } catch (...) {
            std::cout << "uncaught exception of unknown type" << std::endl;
            ++ttgt::current_failures();
        }
        if (ttgt::current_failures()) {
            ++failed;
            std::cout << "[  FAILED  ] " << full << std::endl;
        } else {
            std::cout << "[       OK ] " << full << std::endl;
        }
    }
    std::cout << "[==========] " << run << " tests ran." << std::endl;
    if (failed) {
        std::cout << "[  FAILED  ] " << failed << " tests." << std::endl;
        return 1;
    }
    std::cout << "[  PASSED  ] " << run << " tests." << std::endl;
    return 0;
}
