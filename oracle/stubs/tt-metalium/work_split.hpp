// Empty stand-in: the reference's CPU golden needs no tt-metal work split.
#pragma once
