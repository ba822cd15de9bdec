"""Test infrastructure: the Python restatement of the reference's program
builder, planner and this target's lowering, which the C++ host library
(libfurykernel_host.so) is checked against. Nothing in the package imports
it."""
