"""Import stand-in for vllm-ascend (>=0.25.1rc1,<0.25.2), which is not vendored
in the reference and is not installed here.  Used only by make_golden.py to
import the reference's modules on a host without Ascend hardware."""
