// Empty stand-in: the reference's CPU golden needs no tt-metal host API.
#pragma once
#include <cstdint>
#include <vector>
#include <tuple>
#include <cmath>
#include <iostream>
