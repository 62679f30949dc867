// Test-infrastructure stub (oracle only): the reference's format header includes this;
// none of the host code the oracle compiles uses anything from it.
#pragma once
