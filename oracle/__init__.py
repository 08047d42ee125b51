"""CPU oracle (test infrastructure): a C++ restatement of the reference's hot-path arithmetic."""
