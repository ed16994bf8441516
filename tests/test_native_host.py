"""Host-side behaviour of the native extension that needs no GPU."""
import pytest

from oxidizr_b200.ops._C import raw_ext


def test_failed_launcher_check_raises_python_error():
    e = raw_ext()
    e.host_check_selftest(0)
    with pytest.raises(RuntimeError, match="value 3 of 2.5 true"):
        e.host_check_selftest(3)
