"""The profiling entry point (python -m qw6_b200.prof) parses its command
line without a GPU; the matvec workload itself runs only on a GPU box."""
from qw6_b200 import prof


def test_prof_usage():
    assert prof.main([]) == 2
    assert prof.main(["matvec", "q4k"]) == 2
