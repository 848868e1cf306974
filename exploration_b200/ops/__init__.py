"""Operators: torch reference math and the sm_100a extension behind one interface each."""
