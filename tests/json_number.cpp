// Test helper for tests/test_report_json.py: prints the `diarize` report's JSON form
// (csrc/report_json.h) of each number given as an argument, one per line; with
// --quote, the JSON string form of standard input.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <iterator>
#include <string>

#include "../nemotron3-diarization-wgpu_b200/csrc/report_json.h"

int main(int argc, char** argv) {
    if (argc > 1 && std::strcmp(argv[1], "--quote") == 0) {
        const std::string s((std::istreambuf_iterator<char>(std::cin)), std::istreambuf_iterator<char>());
        std::printf("%s\n", n3d::report::quote(s).c_str());
        return 0;
    }
    for (int i = 1; i < argc; i++) std::printf("%s\n", n3d::report::number(std::strtod(argv[i], nullptr)).c_str());
    return 0;
}
