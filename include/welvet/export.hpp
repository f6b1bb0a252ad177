#pragma once
// Symbol visibility of the C++ layer/volume API exported by libwelvet_b200.so
// (the library is built with hidden visibility; these names are its C++ surface).
#define WELVET_CXX_API __attribute__((visibility("default")))
