// Stand-in for the MUSA runtime header the reference's MSDA kernel header
// includes; the host build of its generic forward kernel needs nothing from
// it (device_shim.h supplies the kernel qualifiers).  TEST INFRASTRUCTURE ONLY.
#pragma once
