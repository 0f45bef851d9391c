"""accel"""
