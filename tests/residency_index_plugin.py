"""pytest plugin (-p residency_index_plugin) that installs the indexed
residency control into the reference package before the reference's own
tests run; used by tests/test_residency_index.py."""

_installed: list = []


def pytest_configure(config):
    import nano_hisparse

    from hisparse_b200 import residency

    _installed[:] = residency.install(nano_hisparse)


def pytest_terminal_summary(terminalreporter):
    terminalreporter.write_line("indexed residency installed: " + ", ".join(_installed))
