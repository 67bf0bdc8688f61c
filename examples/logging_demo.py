"""Logging setup demo (reference: examples/logging_demo.py): console + file, per-module loggers, rank filters."""
import os
import sys
import tempfile

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from nano_train_b200.logging import get_logger, setup_logging, setup_process_logging  # noqa: E402

if __name__ == "__main__":
    log_file = os.path.join(tempfile.mkdtemp(), "demo.log")
    setup_logging(level="DEBUG", log_file=log_file)
    log = get_logger("nano_train_b200.demo")
    log.debug("debug message")
    log.info("info message")
    log.warning("warning message")
    log.error("error message")
    setup_process_logging(rank=1)  # non-zero ranks only show warnings and errors
    get_logger("nano_train_b200.demo").info("hidden on rank 1")
    get_logger("nano_train_b200.demo").warning("shown on rank 1")
    print("log file:", log_file)
    print(open(log_file).read())
