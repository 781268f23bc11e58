"""Data plane (MSHT frames over TCP or pipes) and the HTTP control client."""
