.version 8.0
.target sm_89
.address_size 64

.visible .entry k_row_sumsq_gap(
        .param .u64 param_x,
        .param .u64 param_ss
)
.reqntid 128
{
        .reg .pred      %p<3>;
        .reg .f32       %f<5>;
        .reg .b32       %r<9>;
        .reg .b64       %rd<5>;

        ld.param.u64    %rd1, [param_x];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_ss];
        cvta.to.global.u64     %rd2, %rd2;
        mov.u32         %r1, %tid.x;
        mov.u32         %r2, %ntid.x;
        mov.u32         %r3, %ctaid.x;
        mad.lo.s32      %r4, %r3, %r2, %r1;
        mov.u32         %r5, %nctaid.x;
        setp.ge.s32     %p1, %r4, 17;
        @%p1 bra        SKIP_1;
        mov.f32         %f1, 0f00000000;
        mov.s32         %r6, 0;
        .pragma "nounroll";
LOOP_2:
        mul.lo.s32      %r7, %r4, 300;
        add.s32         %r8, %r7, %r6;
        mad.wide.s32    %rd3, %r8, 4, %rd1;
        ld.global.nc.f32   %f2, [%rd3];
        mul.f32         %f3, %f2, %f2;
        mov.f32         %f4, 0f00000000;
        add.f32         %f1, %f1, %f3;
        add.s32         %r6, %r6, 1;
        setp.lt.s32     %p2, %r6, 300;
        @%p2 bra        LOOP_2;
        mad.wide.s32    %rd4, %r4, 4, %rd2;
        st.global.f32   [%rd4], %f1;
SKIP_1:
        ret;
}
